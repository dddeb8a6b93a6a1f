"""SD3.5 request states and the step-level continuous-batching engine.

Each request owns a seeded latent and a flow-matching solver (Euler by default;
DPM-Solver++ or UniPC on request) over the shifted sigma grid (static shift 3.0,
or the resolution-dependent mu shift).  ``advance_batch(states)``
runs ONE denoising step for every member in a single packed forward (the CFG
branches are two segments of the same request), so requests with different
resolutions and progress join and leave the batch between steps.  Reference:
workers/ditserve/models/sd35.py:816-1164.
"""
from __future__ import annotations

import hashlib
from dataclasses import asdict, dataclass, field

import torch

from ...schedulers import SOLVERS, flow_shift_sigmas, make_scheduler, mu_for_seq_len, scheduler_from_state
from .model import SD35_MEDIUM, SD35Config, SD35Transformer


@dataclass
class SD35Spec:
    height: int = 1024
    width: int = 1024
    steps: int = 28
    guidance: float = 4.5
    seed: int = 0
    text_len: int = 333
    dynamic_shift: bool = False
    prompt: str = ""
    negative_prompt: str = ""
    # "euler" (the SD3.5 default), "dpm++" or "unipc", all on the shifted flow-matching grid
    solver: str = "euler"

    @classmethod
    def normalize(cls, raw: dict) -> "SD35Spec":
        unknown = set(raw) - set(cls.__dataclass_fields__)
        if unknown:
            raise ValueError(f"unknown SD3.5 spec fields: {sorted(unknown)}")
        s = cls(**raw)
        if s.height % 16 or s.width % 16:
            raise ValueError("height and width must be multiples of 16")
        if s.steps < 1:
            raise ValueError("steps must be positive")
        if s.solver not in SOLVERS:
            raise ValueError(f"unknown solver {s.solver!r}; expected one of {SOLVERS}")
        return s

    def to_dict(self):
        return asdict(self)


@dataclass
class SD35State:
    spec: SD35Spec
    latents: torch.Tensor          # fp32 [C, H/8, W/8]
    scheduler: object               # Euler / DPM-Solver++ / UniPC (schedulers package)
    context: torch.Tensor          # [L, joint_dim]
    pooled: torch.Tensor           # [pooled_dim]
    neg_context: torch.Tensor | None
    neg_pooled: torch.Tensor | None
    step: int = 0
    metrics: dict = field(default_factory=dict)

    @property
    def done(self) -> bool:
        return self.step >= self.spec.steps

    def digest(self) -> str:
        return hashlib.sha256(self.latents.detach().cpu().contiguous().numpy().tobytes()).hexdigest()


def synthetic_embeddings(seed: int, length: int, dim: int, pooled_dim: int, which: int):
    """Seeded N(0,1) stand-ins for the CLIP-L/G + T5-XXL outputs (no checkpoints offline)."""
    g = torch.Generator(device="cpu").manual_seed(int(seed) * 2 + which + 0x35)
    return torch.randn(length, dim, generator=g), torch.randn(pooled_dim, generator=g)


class SD35Engine:
    def __init__(self, cfg: SD35Config = SD35_MEDIUM, device="cuda", dtype=torch.bfloat16,
                 model: SD35Transformer | None = None, seed: int = 0, max_batch: int = 8):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.model = model or SD35Transformer.random_init(cfg, device=self.device, dtype=dtype, seed=seed)
        self.max_batch = max_batch

    def prepare(self, spec: SD35Spec | dict, text=None, negative_text=None) -> SD35State:
        """``text`` / ``negative_text``: optional (context [L, joint_dim], pooled [pooled_dim])
        from the text encoders; seeded synthetic embeddings otherwise."""
        spec = spec if isinstance(spec, SD35Spec) else SD35Spec.normalize(spec)
        h, w = spec.height // self.cfg.vae_scale, spec.width // self.cfg.vae_scale
        g = torch.Generator(device="cpu").manual_seed(int(spec.seed))
        lat = torch.randn(self.cfg.in_channels, h, w, generator=g, dtype=torch.float32).to(self.device)
        mu = mu_for_seq_len((h // self.cfg.patch) * (w // self.cfg.patch)) if spec.dynamic_shift else None
        grid = flow_shift_sigmas(spec.steps, self.cfg.shift, mu)
        sched = make_scheduler(spec.solver, spec.steps, sigmas=grid, flow_shift=self.cfg.shift)
        ctx, pool = text or synthetic_embeddings(spec.seed, spec.text_len, self.cfg.joint_dim, self.cfg.pooled_dim, 0)
        nctx = npool = None
        if spec.guidance > 1.0:
            nctx, npool = negative_text or synthetic_embeddings(spec.seed, spec.text_len, self.cfg.joint_dim,
                                                                self.cfg.pooled_dim, 1)
            nctx, npool = nctx.to(self.device, self.dtype), npool.to(self.device, self.dtype)
        return SD35State(spec=spec, latents=lat, scheduler=sched, context=ctx.to(self.device, self.dtype),
                         pooled=pool.to(self.device, self.dtype), neg_context=nctx, neg_pooled=npool)

    @torch.inference_mode()
    def advance_batch(self, states: list) -> list:
        """One denoising step for every unfinished member; finished members are skipped."""
        live = [s for s in states if not s.done]
        if len(live) > self.max_batch:
            raise ValueError(f"continuous batch holds at most {self.max_batch} requests")
        if not live:
            return states
        lats, ts, ctxs, pools, owners = [], [], [], [], []
        for i, s in enumerate(live):
            t = float(s.scheduler.timestep())
            lats.append(s.latents)
            ts.append(t)
            ctxs.append(s.context)
            pools.append(s.pooled)
            owners.append((i, 0))
            if s.neg_context is not None:
                lats.append(s.latents)
                ts.append(t)
                ctxs.append(s.neg_context)
                pools.append(s.neg_pooled)
                owners.append((i, 1))
        preds = self.model.forward_packed(lats, ts, ctxs, pools)
        by_state: dict = {}
        for (i, branch), p in zip(owners, preds):
            by_state.setdefault(i, {})[branch] = p
        for i, s in enumerate(live):
            cond = by_state[i][0]
            uncond = by_state[i].get(1)
            s.scheduler.step(s.latents.view(-1), cond.reshape(-1), None if uncond is None else uncond.reshape(-1),
                             s.spec.guidance)
            s.step += 1
        return states

    def run(self, state: SD35State) -> SD35State:
        while not state.done:
            self.advance_batch([state])
        return state

    def snapshot(self, s: SD35State) -> dict:
        cp = lambda t: None if t is None else t.detach().cpu().clone()
        return dict(kind="sd35_request.v1", spec=s.spec.to_dict(), step=s.step, latents=cp(s.latents),
                    scheduler=s.scheduler.state_dict(), context=cp(s.context), pooled=cp(s.pooled),
                    neg_context=cp(s.neg_context), neg_pooled=cp(s.neg_pooled))

    def restore(self, snap: dict) -> SD35State:
        if snap.get("kind") != "sd35_request.v1":
            raise ValueError("not an SD3.5 request snapshot")
        mv = lambda t: None if t is None else t.to(self.device)
        return SD35State(spec=SD35Spec.normalize(snap["spec"]), latents=mv(snap["latents"]),
                         scheduler=scheduler_from_state(snap["scheduler"], self.device),
                         context=mv(snap["context"]), pooled=mv(snap["pooled"]), neg_context=mv(snap["neg_context"]),
                         neg_pooled=mv(snap["neg_pooled"]), step=int(snap["step"]))
