"""SD3.5 worker backend: atomic requests and step-level continuous batches.

ops: hello, prepare, advance (steps), advance_batch (one denoising step for a list of
state_ids: late joins and early exits allowed), generate_batch (atomic), finish, release,
snapshot, restore.  Reference: workers/ditserve/models/sd35.py:25-1634.
"""
from __future__ import annotations

import time

import torch

from ..base import Backend, progress, transfer_dir
from .model import SD35_MEDIUM, SD35_TINY
from .runtime import SD35Engine, SD35Spec

CONFIGS = {c.name: c for c in (SD35_MEDIUM, SD35_TINY)}


class SD35Backend(Backend):
    operations = Backend.operations + ("advance_batch", "generate_batch", "snapshot", "restore", "inventory",
                                       "block_export", "block_import")

    def __init__(self, config):
        super().__init__(config)
        cfg = CONFIGS[config.get("model", "sd3.5-medium")]
        dev = config.get("device") or ("cuda:0" if torch.cuda.is_available() else "cpu")
        self.device = torch.device(dev)
        dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        self.engine = SD35Engine(cfg, device=self.device, dtype=dtype, seed=int(config.get("seed", 0)),
                                 max_batch=int(config.get("max_batch", 8)))
        self.snapshots: dict = {}

    def capabilities(self):
        return dict(quanta=["step", "atomic"], continuous_batch=self.engine.max_batch, sequence_packing=True,
                    model=self.engine.cfg.name)

    def prepare(self, request):
        key = self.new_id(request)
        spec = {k: v for k, v in request.get("spec", {}).items() if k in SD35Spec.__dataclass_fields__}
        text = negative = None
        enc_cfg = self.config.get("text_encoder")
        if enc_cfg:  # {"config": "tiny" | "full", "seed": n}: CLIP-L + bigG + T5-XXL, seeded weights
            text, negative = self._encode(SD35Spec.normalize(spec), enc_cfg)
        self.states[key] = self.engine.prepare(spec, text=text, negative_text=negative)
        st = self.states[key]
        return dict(state_id=key, progress=progress(st.step, st.spec.steps))

    def _sync(self):
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def advance(self, request):
        st = self.state(request)
        t0 = time.perf_counter()
        for _ in range(min(int(request.get("steps", 1)), st.spec.steps - st.step)):
            self.engine.advance_batch([st])
        self._sync()
        return dict(state_id=request["state_id"], progress=progress(st.step, st.spec.steps),
                    model_ms=(time.perf_counter() - t0) * 1000)

    def advance_batch(self, request):
        ids = list(request["state_ids"])
        states = [self.state(dict(state_id=i)) for i in ids]
        t0 = time.perf_counter()
        self.engine.advance_batch(states)
        self._sync()
        return dict(members=[dict(state_id=i, progress=progress(s.step, s.spec.steps)) for i, s in zip(ids, states)],
                    batch=len(ids), model_ms=(time.perf_counter() - t0) * 1000)

    def generate_batch(self, request):
        out = []
        states = []
        for spec in request["specs"]:
            sid = spec["request_id"]
            self.prepare(dict(id=request["id"], state_id=sid, spec=spec))
            states.append(sid)
        while any(not self.states[s].done for s in states):
            self.engine.advance_batch([self.states[s] for s in states])
        for s in states:
            out.append(self.finish(dict(request, state_id=s)))
            self.release(dict(state_id=s))
        return dict(results=out)

    def _vae(self):
        if getattr(self, "_decoder", None) is None:
            from .vae import SD35VAEDecoder
            dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
            chans = tuple(self.config.get("vae_channels", (128, 256, 512, 512)))
            self._decoder = SD35VAEDecoder.random_init(device=self.device, dtype=dtype,
                                                       seed=int(self.config.get("seed", 0)), channels=chans)
        return self._decoder

    def finish(self, request):
        st = self.state(request)
        if not st.done:
            raise ValueError("request is not complete")
        if request.get("decode", self.config.get("decode_images", False)):
            lat = st.latents if st.latents.dim() == 4 else st.latents[None]
            image = self._vae().decode(lat)
            self._sync()
            art = self.persist(image.float(), request)
            return dict(state_id=request["state_id"], artifact=art, value=art.get("array_sha256"),
                        shape=list(image.shape))
        art = self.persist(st.latents.float(), request)
        return dict(state_id=request["state_id"], artifact=art, value=art.get("array_sha256"))

    def snapshot(self, request):
        st = self.state(request)
        self.snapshots[request["state_id"]] = self.engine.snapshot(st)
        if request.get("mode", "hot") != "keep":
            del self.states[request["state_id"]]
        return dict(state_id=request["state_id"], step=st.step)

    def restore(self, request):
        snap = self.snapshots.pop(request["state_id"], None)
        if snap is None:
            raise ValueError("no snapshot for state_id")
        self.states[request["state_id"]] = self.engine.restore(snap)
        return dict(state_id=request["state_id"])

    def _encode(self, spec, enc_cfg: dict):
        """Prompt and negative prompt through the three encoders; the joint context is cut or
        zero-padded to the spec's text length (77 CLIP positions, then T5)."""
        from ..text_encoders import SD3TextEncoders
        cfg = self.engine.cfg
        if getattr(self, "_text_encoders", None) is None:
            tiny = enc_cfg.get("config", "full") == "tiny"
            dims = None
            if tiny:  # split the tiny model's pooled width 3:5 between CLIP-L and CLIP-G
                wl = cfg.pooled_dim * 3 // 8 // 4 * 4
                dims = (wl, cfg.pooled_dim - wl, cfg.joint_dim)
            dtype = torch.float32 if self.device.type == "cpu" else torch.bfloat16
            self._text_encoders = SD3TextEncoders(tiny=tiny, device=self.device, dtype=dtype,
                                                  seed=int(enc_cfg.get("seed", 0)),
                                                  t5_len=max(1, spec.text_len - 77), tiny_dims=dims)
        enc = self._text_encoders
        if enc.joint_dim != cfg.joint_dim or enc.pooled_dim != cfg.pooled_dim:
            raise ValueError("text encoder widths do not match the model's joint / pooled widths")
        out = []
        for text in (spec.prompt, spec.negative_prompt):
            ctx, pooled = enc(text)
            ctx = ctx[:spec.text_len]
            out.append((ctx.to(self.device, self.engine.dtype), pooled.to(self.device, self.engine.dtype)))
        return out[0], (out[1] if spec.guidance > 1.0 else None)

    def inventory(self, request):
        return dict(states={k: dict(step=v.step, steps=v.spec.steps) for k, v in self.states.items()})

    def block_export(self, request):
        """Step-boundary packet of an image request (host-staged move to another GPU's worker)."""
        import hashlib
        import io
        import os
        from pathlib import Path
        st = self.state(request)
        buf = io.BytesIO()
        torch.save(self.engine.snapshot(st), buf)
        blob = buf.getvalue()
        d = Path(transfer_dir(self.config))
        path = d / f"sd35-packet-{request['state_id']}-{os.getpid()}-{request.get('id', 0)}.pt"
        path.write_bytes(blob)
        return dict(path=str(path), manifest=hashlib.sha256(blob).hexdigest(), bytes=len(blob))

    def block_import(self, request):
        import hashlib
        import io
        import os
        blob = open(request["path"], "rb").read()
        if hashlib.sha256(blob).hexdigest() != request["manifest"]:
            raise ValueError("packet manifest mismatch (tampered or truncated transfer)")
        key = request["state_id"]
        if key in self.states:
            raise ValueError("duplicate live state_id")
        self.states[key] = self.engine.restore(torch.load(io.BytesIO(blob), weights_only=False))
        os.unlink(request["path"])
        st = self.states[key]
        return dict(state_id=key, progress=progress(st.step, st.spec.steps))
