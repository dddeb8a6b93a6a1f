"""Asynchronous VAE decode: one decode stream next to the DiT stream.

``AsyncDecoder.start(latents)`` enqueues the decode of a finished request on a side CUDA
stream (after an event that orders it behind the producing DiT work) and returns a ticket;
``poll(ticket)`` is non-blocking; ``result(ticket)`` waits for the event.  DiT steps of
other requests keep running on the main stream meanwhile (bubble-free decode).  A
``ChunkedDecode`` can also be advanced a few latent frames per call so a long decode
yields the GPU between chunks.  Reference: workers/ditserve/models/wan/async_decode.py:9-89.
"""
from __future__ import annotations

import torch

from .vae import ChunkedDecode, WanVAEDecoder
from .vae_fast import FastChunkedDecode


class AsyncDecoder:
    """On a GPU the decode runs channels-last on the implicit-GEMM tcgen05 convolution
    (``vae_fast``); on the CPU it runs the module's fp32 NCDHW statement.  ``halo`` (a
    ``vae_fast.HaloCL`` over the decode group) splits every frame's rows over the group."""

    def __init__(self, vae: WanVAEDecoder, device):
        self.vae = vae
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.stream = torch.cuda.Stream(self.device) if self.cuda else None
        self.jobs: dict = {}
        self.counter = 0

    def _job(self, z, halo):
        if self.cuda or halo is not None:
            return FastChunkedDecode(self.vae, z, halo)
        return ChunkedDecode(self.vae, z)

    def start(self, latents: torch.Tensor, chunked: bool = False, halo=None) -> str:
        self.counter += 1
        ticket = f"decode-{self.counter}"
        if self.cuda:
            ready = torch.cuda.Event()
            ready.record(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.stream):
                self.stream.wait_event(ready)
                job = self._job(latents.clone(), halo)
                if chunked:
                    self.jobs[ticket] = dict(chunked=job, event=None)
                    return ticket
                out = job.step(1 << 30).result()
                done = torch.cuda.Event()
                done.record(self.stream)
            self.jobs[ticket] = dict(out=out, event=done)
        else:
            job = self._job(latents, halo)
            self.jobs[ticket] = dict(chunked=job, event=None) if chunked else \
                dict(out=job.step(1 << 30).result(), event=None)
        return ticket

    def advance(self, ticket: str, frames: int = 1) -> bool:
        """Advance a chunked decode by ``frames`` latent frames; True once finished."""
        job = self.jobs[ticket]
        dec = job["chunked"]
        if self.cuda:
            with torch.cuda.stream(self.stream):
                dec.step(frames)
                if dec.done:
                    job["out"] = dec.result()
                    job["event"] = torch.cuda.Event()
                    job["event"].record(self.stream)
        else:
            dec.step(frames)
            if dec.done:
                job["out"] = dec.result()
        return dec.done

    def poll(self, ticket: str) -> bool:
        job = self.jobs[ticket]
        if "out" not in job:
            return False
        return job["event"] is None or job["event"].query()

    def result(self, ticket: str) -> torch.Tensor:
        job = self.jobs.pop(ticket)
        if "out" not in job:
            raise RuntimeError("chunked decode not finished")
        if job["event"] is not None:
            job["event"].synchronize()
        return job["out"]
