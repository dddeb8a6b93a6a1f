"""Worker runtime: the JSON-lines server the C++ controller drives, and its host services
(doorbells, GPU occupancy probes, SM partitioning, remote bridge, model integrity)."""
import hashlib
from pathlib import Path

PROTOCOL_VERSION = 1


def file_hash(path, chunk=1 << 20) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(chunk), b""):
            h.update(block)
    return h.hexdigest()


__all__ = ["PROTOCOL_VERSION", "file_hash", "Path"]
