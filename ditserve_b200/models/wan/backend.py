"""Wan worker backend: the JSON op surface over WanEngine.

ops: hello, prepare, advance (steps | blocks | quantum="step", doorbell, check_blocks),
finish, release, snapshot (hot: pinned host copy), restore, block_export / block_import
(continuation packets through a transfer directory, SHA-256 checked), encode_start /
encode_poll (encoder tickets; synthetic UMT5 embeddings offline), distributed (init an
NCCL world and adopt a CFG x SP layout at a step boundary).
Reference: workers/ditserve/models/wan/backend.py:12-652.
"""
from __future__ import annotations

import os
import time
from pathlib import Path

import torch

from ..base import Backend, artifact, progress
from .config import CONFIGS
from .runtime import WanEngine, WanSpec


class WanBackend(Backend):
    operations = Backend.operations + ("snapshot", "restore", "block_export", "block_import", "encode_start",
                                       "encode_poll", "distributed", "inventory", "decode_start", "decode_poll")

    def __init__(self, config):
        super().__init__(config)
        self.model_name = config.get("model", "wan2.1-t2v-1.3b")
        if self.model_name not in CONFIGS:
            raise ValueError(f"unknown Wan model {self.model_name}")
        dev = config.get("device") or ("cuda:0" if torch.cuda.is_available() else "cpu")
        self.device = torch.device(dev)
        dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        self.engine = WanEngine(self.model_name, device=self.device, dtype=dtype, seed=int(config.get("seed", 0)))
        self.snapshots: dict = {}
        self.tickets: dict = {}
        self.transfer_dir = Path(config.get("transfer_dir", "/dev/shm" if os.path.isdir("/dev/shm") else "/tmp"))
        self.layout = None
        self._decoder = None
        self.decodes: dict = {}

    def _async_decoder(self):
        if self._decoder is None:
            from .async_decode import AsyncDecoder
            from .vae import WanVAEDecoder
            dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
            vae = WanVAEDecoder.random_init(device=self.device, dtype=dtype, seed=int(self.config.get("seed", 0)))
            self._decoder = AsyncDecoder(vae, self.device)
        return self._decoder

    def decode_start(self, request):
        """Decode a finished request's latent on the side stream (VAE, Wan2.1 layout)."""
        st = self.state(request)
        if not st.done:
            raise ValueError("decode requires a completed state")
        if self.engine.cfg.in_channels != 16:
            raise ValueError("this backend's VAE decodes 16-channel (Wan2.1) latents")
        dec = self._async_decoder()
        ticket = dec.start(st.latents, chunked=bool(request.get("chunked", False)))
        self.decodes[ticket] = request["state_id"]
        return dict(ticket=ticket, ready=False, state_id=request["state_id"])

    def decode_poll(self, request):
        ticket = request["ticket"]
        if ticket not in self.decodes:
            raise ValueError("unknown decode ticket")
        dec = self._async_decoder()
        if "chunked" in dec.jobs.get(ticket, {}) and "out" not in dec.jobs[ticket]:
            dec.advance(ticket, int(request.get("frames", 1)))
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
        return p

    def prepare(self, request):
        key = self.new_id(request)
        spec = dict(request.get("spec", {}))
        spec.pop("request_id", None)
        spec.setdefault("model", self.model_name)
        spec = {k: v for k, v in spec.items() if k in WanSpec.__dataclass_fields__}
        st = self.engine.prepare(spec)
        self.states[key] = st
        return dict(state_id=key, progress=self._progress(st))

    def advance(self, request):
        st = self.state(request)
        from ...runtime.doorbell import rung
        bell = rung(request)
        t0 = time.perf_counter()
        if request.get("quantum") == "step" or "blocks" in request:
            res = self.engine.advance(st, None if request.get("quantum") == "step" else int(request["blocks"]),
                                      bell=bell, check_every=int(request.get("check_blocks", 1)), timing=True)
        else:
            n = int(request.get("steps", 1))
            res = {}
            for _ in range(min(n, st.spec.steps - st.step)):
                res = self.engine.advance(st, bell=bell, check_every=int(request.get("check_blocks", 1)))
                if res.get("doorbell_stop"):
                    break
        if st.latents.is_cuda:
            torch.cuda.synchronize(st.latents.device)
        res["model_ms"] = (time.perf_counter() - t0) * 1000
        res["progress"] = self._progress(st)
        res["state_id"] = request["state_id"]
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
                from datetime import timedelta
                backend = "nccl" if self.device.type == "cuda" else "gloo"
                dist.init_process_group(backend, init_method=request["init_method"], rank=int(request["rank"]),
                                        world_size=int(request["world_size"]),
                                        timeout=timedelta(seconds=float(request.get("timeout_s", 120))))
            return dict(initialised=True, rank=dist.get_rank(), world_size=dist.get_world_size())
        if action == "layout":
            from ...parallel.layout import FixedLayout, Form
            from ...parallel.runtime import build_parallel
            for st in self.states.values():
                if st.block != 0:
                    raise ValueError("the layout may change only at a solver-step boundary")
            form = Form.parse(request["form"])
            layout = FixedLayout(tuple(request["ranks"]), form, int(request.get("epoch", 0)))
            spec = WanSpec(model=self.model_name, **{k: v for k, v in request.get("spec", {}).items()
                                                     if k in ("height", "width", "frames")})
            lat = spec.latent_shape()
            pctx, plan = build_parallel(layout, dist.get_rank(), self.device, attention=request.get("path", "fused"),
                                        seq_local=self.engine.cfg.tokens(lat) // form.sp, cfg=self.engine.cfg,
                                        pred_numel=lat[0] * lat[1] * lat[2] * lat[3])
            self.engine.pctx, self.engine.cfg_plan = pctx, plan
            self.layout = layout
            return dict(form=form.name, ranks=list(layout.ranks), epoch=layout.epoch)
        if action == "shutdown":
            if dist.is_initialized():
                dist.destroy_process_group()
            return dict(shutdown=True)
        raise ValueError(f"unknown distributed action {action!r}")
