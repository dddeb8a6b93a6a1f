"""Wan request state and step engine.

A request is normalised (H, W multiples of 16, frames = 4k+1), seeded on the
host (CPU generator, so the latent is identical on every device and every SP
degree), and owns a UniPC flow scheduler with device-resident history.  One
``step`` = one DiT forward of both CFG branches (batched as B=2 on one SP
group, or one branch per group under CFG parallelism with a prediction
exchange) followed by the fused CFG+UniPC update.

Reference behaviour: workers/ditserve/models/wan/runtime.py:117-150 (spec),
:603-657 (prepare), :673-720 (step), :784-865 (snapshots).
"""
from __future__ import annotations

import hashlib
import io
from dataclasses import asdict, dataclass, field

import torch

from ...schedulers import SOLVERS, make_scheduler, scheduler_from_state, unipc_flow_sigmas
from .config import CONFIGS, WanConfig
from .model import LocalAttention, WanTransformer


@dataclass
class WanSpec:
    model: str = "wan2.1-t2v-1.3b"
    height: int = 480
    width: int = 832
    frames: int = 81
    steps: int = 50
    guidance: float = 5.0
    seed: int = 0
    flow_shift: float | None = None
    text_len: int | None = None
    prompt: str = ""
    negative_prompt: str = ""
    # approximate mode (opt-in): late-step CFG folding {"warm_frac", "threshold", "fold_span"}
    cfg_fold: dict | None = None
    # "unipc" (the Wan default), "dpm++" (DPM-Solver++ 2M) or "euler", all on the flow-shift grid
    solver: str = "unipc"

    @classmethod
    def normalize(cls, raw: dict) -> "WanSpec":
        known = {f for f in cls.__dataclass_fields__}
        unknown = set(raw) - known
        if unknown:
            raise ValueError(f"unknown Wan spec fields: {sorted(unknown)}")
        spec = cls(**raw)
        if spec.model not in CONFIGS:
            raise ValueError(f"unknown Wan model {spec.model!r}")
        if spec.height % 16 or spec.width % 16:
            raise ValueError("height and width must be multiples of 16")
        if spec.frames < 1 or (spec.frames - 1) % 4:
            raise ValueError("frames must be 4k+1")
        if spec.steps < 1:
            raise ValueError("steps must be positive")
        if spec.solver not in SOLVERS:
            raise ValueError(f"unknown solver {spec.solver!r}; expected one of {SOLVERS}")
        return spec

    def config(self) -> WanConfig:
        return CONFIGS[self.model]

    def latent_shape(self) -> tuple[int, int, int, int]:
        cfg = self.config()
        st, ss, _ = cfg.vae_stride
        return (cfg.in_channels, (self.frames - 1) // st + 1, self.height // ss, self.width // ss)

    def to_dict(self) -> dict:
        return asdict(self)


def synthetic_text(seed: int, length: int, dim: int, which: int) -> torch.Tensor:
    """Seeded N(0,1) text-encoder output standing in for UMT5 (no checkpoint offline)."""
    g = torch.Generator(device="cpu").manual_seed(int(seed) * 2 + which + 0x5eed)
    return torch.randn(1, length, dim, generator=g)


@dataclass
class WanRequestState:
    spec: WanSpec
    latents: torch.Tensor            # fp32 [1, C, F, H, W], device
    scheduler: object               # UniPC / DPM-Solver++ / Euler (schedulers package)
    context: torch.Tensor            # [1, L, text_dim] model dtype, device
    negative: torch.Tensor | None    # [1, L, text_dim] or None (guidance <= 1)
    step: int = 0
    block: int = 0                   # next block inside the current step (block executor)
    packets: dict = field(default_factory=dict)
    metrics: dict = field(default_factory=dict)
    layout_key: tuple | None = None  # layout the current (partial) step runs under
    fold: object | None = None       # CFGFolding state in approximate mode (not snapshotted)

    @property
    def done(self) -> bool:
        return self.step >= self.spec.steps

    def latent_digest(self) -> str:
        return hashlib.sha256(self.latents.detach().cpu().contiguous().numpy().tobytes()).hexdigest()


def _tensor_items(tree, prefix=""):
    if isinstance(tree, torch.Tensor):
        yield prefix, tree.detach().cpu()
    elif isinstance(tree, dict):
        for k in sorted(tree):
            if k == "manifest":
                continue
            yield from _tensor_items(tree[k], f"{prefix}/{k}")
    elif isinstance(tree, (list, tuple)):
        for i, v in enumerate(tree):
            yield from _tensor_items(v, f"{prefix}/{i}")


class CFGLocal:
    """Both CFG branches on this SP group (batched as B = 2)."""

    cfg_size = 1
    cfg_rank = 0

    def exchange(self, pred_mine: torch.Tensor):  # pragma: no cover - unused for local CFG
        raise RuntimeError("no CFG partner")


class WanEngine:
    def __init__(self, cfg: WanConfig | str, device="cuda", dtype=torch.bfloat16, model: WanTransformer | None = None,
                 pctx=None, cfg_plan=None, seed: int = 0):
        self.cfg = CONFIGS[cfg] if isinstance(cfg, str) else cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.model = model or WanTransformer.random_init(self.cfg, device=self.device, dtype=dtype, seed=seed)
        self.model.eval()
        self.pctx = pctx or LocalAttention()
        self.cfg_plan = cfg_plan or CFGLocal()

    # ------------------------------------------------------------------ requests
    def prepare(self, spec: WanSpec | dict, context: torch.Tensor | None = None,
                negative: torch.Tensor | None = None) -> WanRequestState:
        spec = spec if isinstance(spec, WanSpec) else WanSpec.normalize(spec)
        if spec.model != self.cfg.name:
            raise ValueError(f"engine hosts {self.cfg.name}, request wants {spec.model}")
        shape = spec.latent_shape()
        g = torch.Generator(device="cpu").manual_seed(int(spec.seed))
        latents = torch.randn((1, *shape), generator=g, dtype=torch.float32).to(self.device)
        L = spec.text_len or self.cfg.text_len
        if context is None:
            context = synthetic_text(spec.seed, L, self.cfg.text_dim, 0)
        if negative is None and spec.guidance > 1.0:
            negative = synthetic_text(spec.seed, L, self.cfg.text_dim, 1)
        shift = spec.flow_shift or self.cfg.flow_shift
        grid = unipc_flow_sigmas(spec.steps, shift) if spec.solver == "euler" else None  # UniPC's grid
        sched = make_scheduler(spec.solver, spec.steps, sigmas=grid, flow_shift=shift)
        st = WanRequestState(spec=spec, latents=latents, scheduler=sched,
                             context=context.to(self.device, self.dtype),
                             negative=None if negative is None else negative.to(self.device, self.dtype))
        if spec.cfg_fold is not None and st.negative is not None:
            from ..approx import CFGFolding
            st.fold = CFGFolding(spec.steps, **spec.cfg_fold)
        return st

    def branches(self, st: WanRequestState) -> list[int]:
        """CFG branches this rank computes: [0, 1] locally, [cfg_rank] under CFG parallelism."""
        if st.negative is None:
            return [0]
        if self.cfg_plan.cfg_size == 2:
            return [self.cfg_plan.cfg_rank]
        if st.fold is not None and st.fold.fold_now(st.step):
            return [0]  # folded step: the conditional branch only
        return [0, 1]

    def _inputs(self, st: WanRequestState):
        br = self.branches(st)
        ctx = torch.cat([st.context if b == 0 else st.negative for b in br], 0)
        lat = st.latents.expand(len(br), *st.latents.shape[1:])
        t = torch.full((len(br),), float(st.scheduler.timestep()), device=self.device)
        return br, lat, t, ctx

    @torch.inference_mode()
    def predict(self, st: WanRequestState):
        """Velocity predictions (cond, uncond-or-None) of the current step."""
        br, lat, t, ctx = self._inputs(st)
        pred = self.model(lat, t, ctx, self.pctx)
        return self._split(st, br, pred)

    def _split(self, st, br, pred):
        if st.negative is None:
            return pred[0], None
        if st.fold is not None and self.cfg_plan.cfg_size != 2:
            g = st.spec.guidance
            if br == [0]:
                # v = cond + (g-1) d with the last measured d: pass uncond' = cond - d
                st.fold.combine(st.step, g, pred[0], None)
                return pred[0], (pred[0].float() - st.fold.delta.view_as(pred[0])).to(pred[0].dtype)
            st.fold.combine(st.step, g, pred[0], pred[1])
        if len(br) == 2:
            return pred[0], pred[1]
        theirs = self.cfg_plan.exchange(pred[0])
        cond, uncond = (pred[0], theirs) if br[0] == 0 else (theirs, pred[0])
        if st.fold is not None:  # CFG parallelism: both predictions are here after the exchange
            st.fold.observe(st.step, cond.float() - uncond.float())
        return cond, uncond

    @torch.inference_mode()
    def apply(self, st: WanRequestState, cond: torch.Tensor, uncond: torch.Tensor | None):
        st.scheduler.step(st.latents.view(-1), cond.reshape(-1), None if uncond is None else uncond.reshape(-1),
                          st.spec.guidance)
        st.step += 1
        st.block = 0
        st.packets.clear()
        return st

    # ------------------------------------------------------------------ block executor
    def _begin(self, st: WanRequestState):
        if hasattr(self.pctx, "set_step"):
            self.pctx.set_step(st.step, st.spec.steps)  # step-aware collectives (ring codec anchors)
        br, lat, t, ctx = self._inputs(st)
        st.packets["pk"] = self.model.begin(lat, t, ctx, self.pctx)
        st.packets["branches"] = br

    def _finish_step(self, st: WanRequestState):
        pk = st.packets["pk"]
        pred = self.model.predict(pk, self.pctx)
        if st.negative is not None and hasattr(self.cfg_plan, "fused_step"):
            # CFG parallelism over peer memory: exchange + guidance + update in one kernel
            delta = None
            if st.fold is not None:
                delta = torch.empty(st.latents.numel(), device=st.latents.device, dtype=torch.float32)
            step = st.step
            self.cfg_plan.fused_step(st.scheduler, st.latents.view(-1), pred[0], st.spec.guidance, delta_out=delta)
            if delta is not None:
                st.fold.observe(step, delta)
            st.step += 1
            st.block = 0
            st.packets.clear()
            return
        cond, uncond = self._split(st, st.packets["branches"], pred)
        self.apply(st, cond, uncond)

    @torch.inference_mode()
    def advance(self, st: WanRequestState, blocks: int | None = None, *, bell=None, check_every: int = 1,
                group_flag=None, timing: bool = False) -> dict:
        """Run up to ``blocks`` transformer blocks (default: to the end of the current step).

        The quantum never crosses a solver-step boundary.  With a doorbell predicate the
        host enqueues ``check_every`` blocks at a time, waits for the previous interval's
        event (one interval of lead) and stops once the bell has rung; ``group_flag`` (a
        callable taking and returning an int) makes every rank of an SP group agree on the
        stop (MAX over the group) so all ranks stop after the same block.
        """
        if st.done:
            raise RuntimeError("request already finished")
        L = self.cfg.layers
        if not st.packets:
            self._begin(st)
        want = L - st.block if blocks is None else min(int(blocks), L - st.block)
        done = 0
        stopped = False
        prev_evt = None
        t0 = t1 = None
        if timing and st.latents.is_cuda:
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
        pk = st.packets["pk"]
        while done < want:
            chunk = min(max(1, check_every), want - done)
            for _ in range(chunk):
                self.model.forward_block(st.block, pk, self.pctx)
                st.block += 1
                done += 1
            if bell is None or done >= want:
                continue
            evt = None
            if st.latents.is_cuda:
                evt = torch.cuda.Event()
                evt.record()
            if prev_evt is not None:
                prev_evt.synchronize()  # at most one interval of host lead
            prev_evt = evt
            flag = 1 if bell() else 0
            if group_flag is not None:
                flag = group_flag(flag)
            if flag:
                stopped = True
                break
        step_completed = False
        if st.block >= L:
            self._finish_step(st)
            step_completed = True
        out = dict(blocks=done, next_block=st.block, step_completed=step_completed, doorbell_stop=stopped,
                   step=st.step, steps=st.spec.steps)
        if t0 is not None:
            t1.record()
            t1.synchronize()
            out["block_cuda_ms"] = t0.elapsed_time(t1)
        return out

    @torch.inference_mode()
    def advance_pair(self, a: WanRequestState, b: WanRequestState, blocks: int | None = None, *, bell=None,
                     check_every: int = 1, group_flag=None) -> dict:
        """Lockstep interleave of two requests on one group: block i of ``a``, then block i of
        ``b``, for up to ``blocks`` block pairs, stopping at either request's step boundary or
        at the doorbell (checked every ``check_every`` pairs, group-agreed via ``group_flag``).
        One quantum advances both requests, which is what the planner prices as a pair.
        Reference: advance_pair, workers/ditserve/models/wan/block.py:695-810.
        """
        for st in (a, b):
            if st.done:
                raise RuntimeError("request already finished")
            if not st.packets:
                self._begin(st)
        L = self.cfg.layers
        want = min(L - a.block, L - b.block) if blocks is None else min(int(blocks), L - a.block, L - b.block)
        done, stopped = 0, False
        while done < want:
            for _ in range(min(max(1, check_every), want - done)):
                for st in (a, b):
                    self.model.forward_block(st.block, st.packets["pk"], self.pctx)
                    st.block += 1
                done += 1
            if bell is None or done >= want:
                continue
            flag = 1 if bell() else 0
            if group_flag is not None:
                flag = group_flag(flag)
            if flag:
                stopped = True
                break
        out = {}
        for key, st in (("a", a), ("b", b)):
            completed = st.block >= L
            if completed:
                self._finish_step(st)
            out[key] = dict(next_block=st.block, step_completed=completed, step=st.step, steps=st.spec.steps)
        out.update(blocks=done, doorbell_stop=stopped)
        return out

    def step(self, st: WanRequestState) -> WanRequestState:
        if st.done:
            raise RuntimeError("request already finished")
        self.advance(st)
        return st

    def run(self, st: WanRequestState, steps: int | None = None) -> WanRequestState:
        n = st.spec.steps - st.step if steps is None else steps
        for _ in range(n):
            self.step(st)
        return st

    # ------------------------------------------------------------------ snapshots
    def snapshot(self, st: WanRequestState, device="cpu") -> dict:
        """Exact request state (latents + solver history + text) on ``device`` (pinned when CPU)."""
        def mv(t):
            if t is None:
                return None
            out = t.detach().to(device, copy=True)
            return out.pin_memory() if str(device) == "cpu" and torch.cuda.is_available() else out
        return dict(kind="wan_request.v1", spec=st.spec.to_dict(), step=st.step, latents=mv(st.latents),
                    context=mv(st.context), negative=mv(st.negative),
                    scheduler=st.scheduler.state_dict(device=device))

    def restore(self, snap: dict) -> WanRequestState:
        if snap.get("kind") != "wan_request.v1":
            raise ValueError("not a Wan request snapshot")
        spec = WanSpec.normalize(snap["spec"])
        st = WanRequestState(spec=spec, latents=snap["latents"].to(self.device, copy=True),
                             scheduler=scheduler_from_state(snap["scheduler"], self.device),
                             context=snap["context"].to(self.device, copy=True),
                             negative=None if snap["negative"] is None else snap["negative"].to(self.device, copy=True),
                             step=int(snap["step"]))
        if spec.cfg_fold is not None and st.negative is not None:
            from ..approx import CFGFolding
            st.fold = CFGFolding(spec.steps, **spec.cfg_fold)  # the gate restarts: no delta yet
        return st

    def export_packet(self, st: WanRequestState) -> tuple[bytes, str]:
        """Serialise a request mid-step (continuation packet) with a SHA-256 manifest."""
        snap = self.snapshot(st)
        snap["block"] = st.block
        if st.packets:
            pk = st.packets["pk"]
            snap["packet"] = {k: v.detach().cpu().clone() for k, v in pk.tensors().items()}
            snap["packet_meta"] = dict(batch=pk.batch, seq_local=pk.seq_local, seq=pk.seq, grid=list(pk.grid),
                                       text_len=pk.text_len, next_block=pk.next_block,
                                       branches=list(st.packets["branches"]))
        manifest = {}
        for name, t in _tensor_items(snap):
            manifest[name] = hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()
        snap["manifest"] = manifest
        blob = self.pack(snap)
        return blob, hashlib.sha256(blob).hexdigest()

    def import_packet(self, blob: bytes, digest: str) -> WanRequestState:
        if hashlib.sha256(blob).hexdigest() != digest:
            raise ValueError("packet digest mismatch (tampered or truncated transfer)")
        snap = self.unpack(blob)
        manifest = snap.pop("manifest")
        for name, t in _tensor_items(snap):
            if hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest() != manifest.get(name):
                raise ValueError(f"tensor {name} does not match its manifest")
        st = self.restore(snap)
        st.block = int(snap.get("block", 0))
        if "packet" in snap:
            from .model import WanPacket
            meta = snap["packet_meta"]
            t = {k: v.to(self.device) for k, v in snap["packet"].items()}
            cos_full, sin_full = self.model.rope(tuple(meta["grid"]), self.device)
            pk = WanPacket(x=t["x"], mod=t["mod"], temb=t["temb"], ctx=t["ctx"], cos=t["cos"], sin=t["sin"],
                           batch=meta["batch"], seq_local=meta["seq_local"], seq=meta["seq"], grid=tuple(meta["grid"]),
                           text_len=meta["text_len"], next_block=meta["next_block"], cos_full=cos_full,
                           sin_full=sin_full)
            st.packets = {"pk": pk, "branches": meta["branches"]}
        return st

    @staticmethod
    def pack(snap: dict) -> bytes:
        buf = io.BytesIO()
        torch.save(snap, buf)
        return buf.getvalue()

    @staticmethod
    def unpack(data: bytes) -> dict:
        return torch.load(io.BytesIO(data), weights_only=False)
