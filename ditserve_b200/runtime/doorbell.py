"""Doorbells: asynchronous, RPC-free stop requests from the controller.

One 8-byte little-endian epoch counter per GPU in an mmap'd file.  The
controller rings by writing a larger epoch (the C++ side uses pwrite); a
worker running a block quantum records the epoch current at dispatch and stops
at its next check once the file holds a larger value.  Reference:
workers/ditserve/runtime/doorbell.py:18-61.
"""
from __future__ import annotations

import mmap
import os
import struct


class Doorbell:
    SIZE = 8

    def __init__(self, path: str, create: bool = False):
        self.path = path
        flags = os.O_RDWR | (os.O_CREAT if create else 0)
        self.fd = os.open(path, flags, 0o644)
        if os.fstat(self.fd).st_size < self.SIZE:
            os.ftruncate(self.fd, self.SIZE)
        self.map = mmap.mmap(self.fd, self.SIZE)

    def epoch(self) -> int:
        return struct.unpack_from("<Q", self.map, 0)[0]

    def ring(self, epoch: int | None = None) -> int:
        value = self.epoch() + 1 if epoch is None else int(epoch)
        struct.pack_into("<Q", self.map, 0, value)
        self.map.flush()
        return value

    def close(self):
        try:
            self.map.close()
        finally:
            os.close(self.fd)


def rung(request: dict):
    """Return a zero-argument predicate for ``request["doorbell"] = {path, epoch}``,
    true once the bell's epoch exceeds the dispatch epoch; None without a doorbell."""
    spec = request.get("doorbell")
    if not spec:
        return None
    bell = Doorbell(spec["path"])
    start = int(spec.get("epoch", 0))

    def check() -> bool:
        return bell.epoch() > start

    return check
