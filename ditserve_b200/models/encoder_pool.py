"""Prompt path: proactive text-encoder pool with /dev/shm staging and a negative-prompt cache.

* ``EncoderPool`` runs text encoding on a background thread as soon as a request is
  announced (``submit`` returns a ticket); results are staged in shared-memory slabs
  (``/dev/shm`` .npy files, visible to every worker process on the node) and fetched by
  any worker with ``fetch(ticket)`` — then copied to the GPU from pinned memory.
* Encoders are pluggable callables ``encode(prompt, max_len) -> (tokens [L, dim], valid)``.
  Offline there are no UMT5/CLIP/T5 checkpoints, so ``SyntheticEncoder`` produces seeded
  N(0, 1) embeddings keyed by the prompt text (same prompt -> same embedding).
* ``trim_and_pad``: encode only the valid tokens and zero-pad to ``max_len`` — the
  encoder output is identical to encoding the padded sequence under an attention mask,
  at a fraction of the encoder cost (the reference's UMT5 valid-token crop).
* ``NegativePromptCache``: LRU bounded by entries and bytes (negative prompts repeat).
Reference: workers/ditserve/models/encoder_pool.py:41-471, wan/prompt_cache.py:41-139.
"""
from __future__ import annotations

import hashlib
import os
import queue
import tempfile
import threading
from collections import OrderedDict
from pathlib import Path

import numpy as np
import torch


class SyntheticEncoder:
    def __init__(self, dim: int, tokens_per_word: int = 1):
        self.dim = dim
        self.tokens_per_word = tokens_per_word

    def __call__(self, prompt: str, max_len: int):
        valid = max(1, min(max_len, len(prompt.split()) * self.tokens_per_word))
        seed = int(hashlib.sha256(prompt.encode()).hexdigest()[:8], 16)
        g = torch.Generator().manual_seed(seed)
        return torch.randn(valid, self.dim, generator=g), valid


def trim_and_pad(tokens: torch.Tensor, valid: int, max_len: int) -> torch.Tensor:
    out = torch.zeros(max_len, tokens.shape[-1], dtype=tokens.dtype)
    out[:valid] = tokens[:valid]
    return out


class NegativePromptCache:
    def __init__(self, max_entries: int = 16, max_bytes: int = 256 << 20):
        self.max_entries, self.max_bytes = max_entries, max_bytes
        self.items: OrderedDict = OrderedDict()
        self.bytes = 0
        self.hits = self.misses = 0

    def get(self, key):
        if key in self.items:
            self.items.move_to_end(key)
            self.hits += 1
            return self.items[key]
        self.misses += 1
        return None

    def put(self, key, value: torch.Tensor):
        nb = value.numel() * value.element_size()
        if nb > self.max_bytes:
            return
        if key in self.items:
            self.bytes -= self.items.pop(key).numel() * value.element_size()
        self.items[key] = value
        self.bytes += nb
        while len(self.items) > self.max_entries or self.bytes > self.max_bytes:
            _, old = self.items.popitem(last=False)
            self.bytes -= old.numel() * old.element_size()


class EncoderPool:
    def __init__(self, encoder, max_len: int, slab_dir: str | None = None, negative_cache: NegativePromptCache | None = None):
        self.encoder = encoder
        self.max_len = max_len
        base = slab_dir or ("/dev/shm" if os.path.isdir("/dev/shm") else tempfile.gettempdir())
        self.dir = Path(tempfile.mkdtemp(prefix="ds-encpool-", dir=base))
        self.neg = negative_cache or NegativePromptCache()
        self.q: queue.Queue = queue.Queue()
        self.done: dict = {}
        self.cv = threading.Condition()
        self.counter = 0
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _encode(self, prompt: str) -> np.ndarray:
        tokens, valid = self.encoder(prompt, self.max_len)
        return trim_and_pad(tokens, valid, self.max_len).float().numpy()

    def _run(self):
        while True:
            item = self.q.get()
            if item is None:
                return
            ticket, prompt, negative = item
            try:
                pos = self._encode(prompt)
                neg = None
                if negative is not None:
                    cached = self.neg.get(negative)
                    if cached is None:
                        cached = torch.from_numpy(self._encode(negative))
                        self.neg.put(negative, cached)
                    neg = cached.numpy()
                paths = {}
                for name, arr in (("prompt", pos), ("negative", neg)):
                    if arr is None:
                        continue
                    p = self.dir / f"{ticket}-{name}.npy"
                    np.save(p, arr, allow_pickle=False)
                    paths[name] = str(p)
                result = dict(ready=True, paths=paths)
            except Exception as exc:  # noqa: BLE001 - reported to the fetching worker
                result = dict(ready=True, error=str(exc))
            with self.cv:
                self.done[ticket] = result
                self.cv.notify_all()

    def submit(self, prompt: str, negative: str | None = None) -> str:
        with self.cv:
            self.counter += 1
            ticket = f"enc-{os.getpid()}-{self.counter}"
        self.q.put((ticket, prompt, negative))
        return ticket

    def poll(self, ticket: str) -> bool:
        with self.cv:
            return ticket in self.done

    def fetch(self, ticket: str, device=None, dtype=torch.bfloat16, timeout: float = 60.0):
        with self.cv:
            if not self.cv.wait_for(lambda: ticket in self.done, timeout=timeout):
                raise TimeoutError(f"encode ticket {ticket} not ready")
            res = self.done.pop(ticket)
        if "error" in res:
            raise RuntimeError(res["error"])
        out = {}
        for name, p in res["paths"].items():
            arr = torch.from_numpy(np.load(p, mmap_mode="r").copy())
            if device is not None and torch.device(device).type == "cuda":
                arr = arr.pin_memory().to(device, dtype, non_blocking=True)
            else:
                arr = arr.to(dtype)
            out[name] = arr
            os.unlink(p)
        return out

    def close(self):
        self.q.put(None)
        self.t.join(timeout=5)
        for p in self.dir.glob("*"):
            p.unlink()
        self.dir.rmdir()
