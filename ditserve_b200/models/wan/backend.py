"""Wan worker backend: the JSON op surface over WanEngine.

ops: hello, prepare, advance (steps | blocks | quantum="step", doorbell, check_blocks),
finish, release, snapshot (hot: pinned host copy), restore, block_export / block_import
(continuation packets through a transfer directory, SHA-256 checked), encode_start /
encode_poll (encoder tickets; synthetic UMT5 embeddings offline), decode_start / decode_poll
(VAE decode on a side stream, optionally chunked), advance_pair (lockstep pair quantum),
distributed (init an NCCL world; adopt a CFG x SP layout at a step boundary; group
consensus; regroup state broadcast over peer memory or NCCL; shutdown).
Reference: workers/ditserve/models/wan/backend.py:12-652.
"""
from __future__ import annotations

import json
import math
import os
import time
from pathlib import Path

import torch

from ..base import Backend, progress, transfer_dir
from .config import CONFIGS
from .runtime import WanEngine, WanSpec


def decode_halo_transport(choice: str, members: int, device_type: str) -> str:
    """Halo transport of a patch-parallel VAE decode: ``peer`` (stores into the neighbours' heap
    slots, one group barrier per convolution) or ``nccl`` (send/recv).  ``auto`` takes peer
    memory for two members and send/recv beyond: 480p 81-frame decodes measured 613 vs 648 ms on
    two B200s and 362 vs 349 ms on four, where the per-convolution barrier over four ranks costs
    more than the stores save.  Off the GPU it is always send/recv."""
    if choice not in ("auto", "peer", "nccl"):
        raise ValueError(f"decode_halo must be auto, peer or nccl, not {choice!r}")
    if device_type != "cuda":
        return "nccl"
    if choice == "auto":
        return "peer" if members <= 2 else "nccl"
    return choice


class WanBackend(Backend):
    operations = Backend.operations + ("snapshot", "restore", "block_export", "block_import", "encode_start",
                                       "encode_poll", "distributed", "inventory", "decode_start", "decode_poll",
                                       "advance_pair")

    def __init__(self, config):
        super().__init__(config)
        self.model_name = config.get("model", "wan2.1-t2v-1.3b")
        if self.model_name not in CONFIGS:
            raise ValueError(f"unknown Wan model {self.model_name}")
        dev = config.get("device") or ("cuda:0" if torch.cuda.is_available() else "cpu")
        self.device = torch.device(dev)
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)  # NCCL and the object collectives use the current device
        dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        self.engine = WanEngine(self.model_name, device=self.device, dtype=dtype, seed=int(config.get("seed", 0)))
        self.snapshots: dict = {}
        self.tickets: dict = {}
        self.transfer_dir = Path(transfer_dir(config))
        self.layout = None
        self._decoder = None
        self._decode_halos: dict = {}
        self.decodes: dict = {}
        self._comm: dict = {}
        self._layouts: dict = {}
        self.group_flag = None

    def _group(self, request):
        """Process group over request['ranks'] (member-local creation, cached per rank set)."""
        import torch.distributed as dist
        from ...parallel.runtime import group_for
        return group_for(request.get("ranks", range(dist.get_world_size())))

    def _adopt(self, request, st=None):
        """Make ``request``'s layout {ranks, form, epoch, spec, path} current.

        Built plans are cached per (ranks, form, latent shape, path): switching between
        requests of different layouts is a lookup.  A request inside a solver step keeps the
        layout its step started with.
        """
        import torch.distributed as dist
        from ...parallel.layout import FixedLayout, Form
        form = Form.parse(request["form"])
        ranks = tuple(int(r) for r in request["ranks"])
        if st is not None:
            shape = tuple(st.latents.shape[1:])
        else:
            spec = WanSpec(model=self.model_name, **{k: v for k, v in request.get("spec", {}).items()
                                                     if k in ("height", "width", "frames")})
            shape = tuple(spec.latent_shape())
        path = request.get("path", "fused")
        if path == "auto":  # measured choice per (form, tokens per rank)
            from ...parallel.autotune import choose
            path = choose(form.name, self.engine.cfg.tokens(shape) // form.sp)
        key = (ranks, form.name, shape, path)
        if path == "nccl-fp8" and request.get("fp8_layers") is not None:
            key += (tuple(sorted(int(i) for i in request["fp8_layers"])),)
        codec = request.get("ring_codec", self.config.get("ring_codec"))
        if codec is not None and form.ring > 1:
            key += (("ring_codec", json.dumps(codec, sort_keys=True)),)
        if st is not None and st.block != 0 and st.layout_key not in (None, key):
            raise ValueError("the SP group may change only at a solver-step boundary")
        if key not in self._layouts:
            layout = FixedLayout(ranks, form, int(request.get("epoch", 0)))
            if form.gpus == 1:
                from .model import LocalAttention
                from .runtime import CFGLocal
                self._layouts[key] = (layout, LocalAttention(), CFGLocal(), None)
            else:
                from ...parallel.elastic import GroupFlagNCCL, GroupFlagPeer
                from ...parallel.runtime import build_parallel, group_for
                rank = dist.get_rank()
                pctx, plan = build_parallel(layout, rank, self.device, attention=path,
                                            seq_local=self.engine.cfg.tokens(shape) // form.sp, cfg=self.engine.cfg,
                                            pred_numel=math.prod(shape), fp8_layers=request.get("fp8_layers"),
                                            ring_codec=codec)
                flag = None
                if form.sp > 1:  # doorbell stop agreed over the SP group (MAX of the ranks' flags)
                    sp = layout.sp_ranks(rank)
                    g = group_for(sp)
                    if path == "fused" and self.device.type == "cuda":
                        from ...parallel.symm import SymmetricHeap
                        heap = SymmetricHeap(1 << 20, self.device, group=g)
                        flag = GroupFlagPeer(heap, tuple(range(len(sp))))
                    else:
                        flag = GroupFlagNCCL(g, self.device)
                self._layouts[key] = (layout, pctx, plan, flag)
        layout, pctx, plan, flag = self._layouts[key]
        self.engine.pctx, self.engine.cfg_plan, self.group_flag = pctx, plan, flag
        self.layout = layout
        if st is not None:
            st.layout_key = key
        return key

    def _async_decoder(self):
        if self._decoder is None:
            from .async_decode import AsyncDecoder
            from .vae import WanVAEDecoder
            dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
            variant = "wan2.2" if self.engine.cfg.in_channels == 48 else "wan2.1"
            vae = WanVAEDecoder.random_init(device=self.device, dtype=dtype, seed=int(self.config.get("seed", 0)),
                                            variant=variant)
            self._decoder = AsyncDecoder(vae, self.device)
        return self._decoder

    def _decode_halo(self, group):
        """Row halo of a patch-parallel decode over ``group`` (global ranks), cached per group:
        peer-memory stores into the neighbours' halo slots or send/recv (decode_halo_transport)."""
        key = tuple(sorted(int(r) for r in group))
        if key not in self._decode_halos:
            from ...parallel.runtime import group_for
            from .vae_fast import NCCLHaloCL, PeerHaloCL
            g = group_for(key)
            if decode_halo_transport(self.config.get("decode_halo", "auto"), len(key), self.device.type) == "peer":
                from ...parallel.fused import PeerHalo
                from ...parallel.symm import SymmetricHeap
                elems = int(self.config.get("decode_halo_elems", 4 << 20))
                heap = SymmetricHeap(4 * elems * 4 + (1 << 20), self.device, group=g)
                halo = PeerHaloCL(PeerHalo(heap, tuple(range(len(key))), max_halo_elems=elems), group=g)
            else:
                halo = NCCLHaloCL(g)
            self._decode_halos[key] = halo
        return self._decode_halos[key]

    def decode_start(self, request):
        """Decode a finished request's latent on the side stream (Wan2.1 or Wan2.2 VAE).

        With ``group`` (global ranks, every member calling with the same request) the decode is
        patch parallel: each member decodes its rows of every frame, completing each 3-high
        convolution's input with one halo row from each neighbour, and the finished video is
        gathered on every member."""
        st = self.state(request)
        if not st.done:
            raise ValueError("decode requires a completed state")
        if self.engine.cfg.in_channels not in (16, 48):
            raise ValueError("no VAE for this latent width")
        dec = self._async_decoder()
        group = request.get("group")
        halo = self._decode_halo(group) if group is not None and len(group) > 1 else None
        ticket = dec.start(st.latents, chunked=bool(request.get("chunked", False)), halo=halo)
        self.decodes[ticket] = request["state_id"]
        return dict(ticket=ticket, ready=False, state_id=request["state_id"])

    def decode_poll(self, request):
        ticket = request["ticket"]
        if ticket not in self.decodes:
            raise ValueError("unknown decode ticket")
        dec = self._async_decoder()
        if "chunked" in dec.jobs.get(ticket, {}) and "out" not in dec.jobs[ticket]:
            # a waiting poll finishes the decode whatever frame count it names
            frames = 1 << 30 if request.get("wait") else int(request.get("frames", 1))
            dec.advance(ticket, frames)
        if not dec.poll(ticket) and not request.get("wait"):
            return dict(ticket=ticket, ready=False)
        video = dec.result(ticket)
        sid = self.decodes.pop(ticket)
        art = self.persist(video.float(), dict(request, state_id=sid))
        return dict(ticket=ticket, ready=True, state_id=sid, artifact=art, shape=list(video.shape))

    def capabilities(self):
        return dict(quanta=["step", "blocks"], blocks_per_step=self.engine.cfg.layers, migration=True,
                    sp_degrees=[1, 2, 3, 4, 6, 8], model=self.model_name, device=str(self.device))

    def _progress(self, st):
        p = progress(st.step, st.spec.steps)
        p["block"] = st.block
        p["transfer_ready"] = st.block == 0
        if st.fold is not None:
            p["cfg_fold_eligible"] = bool(st.block == 0 and not st.done and st.fold.eligible(st.step))
        return p

    def prepare(self, request):
        key = self.new_id(request)
        spec = dict(request.get("spec", {}))
        spec.pop("request_id", None)
        spec.setdefault("model", self.model_name)
        spec = {k: v for k, v in spec.items() if k in WanSpec.__dataclass_fields__}
        context = negative = None
        enc_cfg = self.config.get("text_encoder")
        if enc_cfg:  # {"config": "tiny" | "xxl", "seed": n}: UMT5 architecture, seeded weights
            context, negative = self._encode(WanSpec.normalize(spec), enc_cfg)
        st = self.engine.prepare(spec, context=context, negative=negative)
        self.states[key] = st
        return dict(state_id=key, progress=self._progress(st))

    def _encode(self, spec: WanSpec, enc_cfg: dict):
        """Prompt and negative prompt through the UMT5 encoder: valid tokens only, zero-padded
        to the model's text length (the valid-token crop)."""
        from ..encoder_pool import trim_and_pad
        from ..text_encoders import TINY_T5, UMT5TextEncoder
        if getattr(self, "_text_encoder", None) is None:
            cfg = TINY_T5 if enc_cfg.get("config", "xxl") == "tiny" else None
            dtype = torch.float32 if self.device.type == "cpu" else torch.bfloat16
            self._text_encoder = UMT5TextEncoder(cfg, device=self.device, dtype=dtype,
                                                 seed=int(enc_cfg.get("seed", 0)))
        L = spec.text_len or self.engine.cfg.text_len
        if self._text_encoder.dim != self.engine.cfg.text_dim:
            raise ValueError(f"text encoder width {self._text_encoder.dim} != model text_dim {self.engine.cfg.text_dim}")
        out = []
        for text in (spec.prompt, spec.negative_prompt):
            tokens, valid = self._text_encoder(text, L)
            out.append(trim_and_pad(tokens, valid, L)[None])
        return out[0], (out[1] if spec.guidance > 1.0 else None)

    def advance(self, request):
        if request.get("pair_state_id") is not None:
            return self.advance_pair(dict(request, state_ids=[request["state_id"], request["pair_state_id"]]))
        st = self.state(request)
        if request.get("layout") is not None:
            self._adopt(request["layout"], st)
        from ...runtime.doorbell import rung
        bell = rung(request)
        t0 = time.perf_counter()
        if request.get("quantum") == "step" or "blocks" in request:
            res = self.engine.advance(st, None if request.get("quantum") == "step" else int(request["blocks"]),
                                      bell=bell, check_every=int(request.get("check_blocks", 1)), timing=True,
                                      group_flag=self.group_flag)
        else:
            n = int(request.get("steps", 1))
            res = {}
            for _ in range(min(n, st.spec.steps - st.step)):
                res = self.engine.advance(st, bell=bell, check_every=int(request.get("check_blocks", 1)),
                                          group_flag=self.group_flag)
                if res.get("doorbell_stop"):
                    break
        if st.latents.is_cuda:
            torch.cuda.synchronize(st.latents.device)
        res["model_ms"] = (time.perf_counter() - t0) * 1000
        res["progress"] = self._progress(st)
        res["state_id"] = request["state_id"]
        return res

    def advance_pair(self, request):
        """Lockstep pair quantum: ``state_ids`` [a, b], up to ``blocks`` block pairs."""
        from ...runtime.doorbell import rung
        ida, idb = request["state_ids"]
        if ida == idb:
            raise ValueError("a pair needs two distinct states")
        a, b = self.state(dict(state_id=ida)), self.state(dict(state_id=idb))
        if request.get("layout") is not None:
            self._adopt(request["layout"], a)
            self._adopt(request["layout"], b)
        t0 = time.perf_counter()
        blocks = request.get("blocks")
        res = self.engine.advance_pair(a, b, None if blocks is None else int(blocks), bell=rung(request),
                                       check_every=int(request.get("check_blocks", 1)), group_flag=self.group_flag)
        if a.latents.is_cuda:
            torch.cuda.synchronize(a.latents.device)
        res["model_ms"] = (time.perf_counter() - t0) * 1000
        res["a"].update(state_id=ida, progress=self._progress(a))
        res["b"].update(state_id=idb, progress=self._progress(b))
        res["state_id"], res["progress"] = ida, res["a"]["progress"]
        res["pair_state_id"], res["pair_progress"] = idb, res["b"]["progress"]
        return res

    def finish(self, request):
        st = self.state(request)
        if not st.done:
            raise ValueError("request is not complete")
        art = self.persist(st.latents.float(), request)
        return dict(state_id=request["state_id"], artifact=art, value=art.get("array_sha256"))

    def snapshot(self, request):
        st = self.state(request)
        mode = request.get("mode", "hot")
        self.snapshots[request["state_id"]] = self.engine.snapshot(st, device="cpu")
        if mode in ("hot", "cold"):
            del self.states[request["state_id"]]
        return dict(state_id=request["state_id"], mode=mode, step=st.step)

    def restore(self, request):
        sid = request["state_id"]
        snap = self.snapshots.pop(sid, None)
        if snap is None:
            raise ValueError("no snapshot for state_id")
        self.states[sid] = self.engine.restore(snap)
        return dict(state_id=sid, progress=self._progress(self.states[sid]))

    def block_export(self, request):
        st = self.state(request)
        blob, digest = self.engine.export_packet(st)
        path = self.transfer_dir / f"wan-packet-{request['state_id']}-{os.getpid()}-{request['id']}.pt"
        path.write_bytes(blob)
        return dict(path=str(path), manifest=digest, bytes=len(blob))

    def block_import(self, request):
        blob = Path(request["path"]).read_bytes()
        st = self.engine.import_packet(blob, request["manifest"])
        key = request.get("state_id") or self.new_id(dict(spec={"request_id": request["state_id"]}))
        if key in self.states:
            raise ValueError("duplicate live state_id")
        self.states[key] = st
        Path(request["path"]).unlink(missing_ok=True)  # a packet is single-use (one export per hop)
        return dict(state_id=key, progress=self._progress(st))

    def encode_start(self, request):
        ticket = f"encode-{request['id']}"
        self.tickets[ticket] = dict(request.get("spec", {}))
        return dict(ticket=ticket, ready=True, synthetic=True)

    def encode_poll(self, request):
        if request["ticket"] not in self.tickets:
            raise ValueError("unknown encode ticket")
        return dict(ticket=request["ticket"], ready=True)

    def inventory(self, request):
        return dict(states={k: dict(step=v.step, block=v.block, steps=v.spec.steps) for k, v in self.states.items()},
                    snapshots=sorted(self.snapshots))

    def distributed(self, request):
        """action=init: join an NCCL world; action=layout: adopt a CFG x SP form (step boundary only)."""
        import torch.distributed as dist
        action = request.get("action", "init")
        if action == "init":
            if not dist.is_initialized():
                # lazy communicator init (no device_id): sub-groups are then created by their
                # members alone instead of by a split that every world rank must join
                from datetime import timedelta
                backend = "nccl" if self.device.type == "cuda" else "gloo"
                dist.init_process_group(backend, init_method=request["init_method"], rank=int(request["rank"]),
                                        world_size=int(request["world_size"]),
                                        timeout=timedelta(seconds=float(request.get("timeout_s", 120))))
            return dict(initialised=True, rank=dist.get_rank(), world_size=dist.get_world_size())
        if action == "layout":
            for st in self.states.values():
                if st.block != 0:
                    raise ValueError("the layout may change only at a solver-step boundary")
            key = self._adopt(request)
            return dict(form=key[1], ranks=list(key[0]), epoch=self.layout.epoch)
        if action == "consensus":
            from ...parallel.elastic import RequestGroupGate, state_digest
            group = self._group(request)
            sid = request["state_id"]
            st = self.states[sid]
            agreed = RequestGroupGate(group).consensus(state_digest(sid, st, int(request.get("epoch", 0))))
            return dict(state_id=sid, agreed=agreed, step=st.step, block=st.block)
        if action == "migrate_group":
            # regroup: the source rank's state reaches every rank of the new group, bit-exact
            from ...parallel.elastic import PeerStateBroadcast, broadcast_state_nccl
            ranks = tuple(int(r) for r in request["ranks"])
            src = int(request["src"])
            sid = request["state_id"]
            me = dist.get_rank()
            tree = None
            if me == src:
                st = self.states[sid]
                if st.block != 0:
                    raise ValueError("regroup only at a solver-step boundary")
                tree = self.engine.snapshot(st, device=self.device)
            group = self._group(request)
            if request.get("path", "fused") == "fused" and self.device.type == "cuda":
                key = ("bcast", ranks)
                if key not in self._comm:
                    from ...parallel.symm import SymmetricHeap
                    cap = int(request.get("capacity_mb", 256)) << 20
                    heap = SymmetricHeap(cap + (1 << 20), self.device, group=group)
                    self._comm[key] = PeerStateBroadcast(heap, tuple(range(len(ranks))), cap, group=group)
                tree = self._comm[key](tree, ranks.index(src), src)
            else:
                tree = broadcast_state_nccl(tree, src, group=group, device=self.device)
            if me != src:
                self.states[sid] = self.engine.restore(tree)
            st = self.states[sid]
            return dict(state_id=sid, step=st.step, ranks=list(ranks))
        if action == "shutdown":
            if dist.is_initialized():
                dist.destroy_process_group()
            return dict(shutdown=True)
        raise ValueError(f"unknown distributed action {action!r}")
