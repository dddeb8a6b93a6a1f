"""Backend contract: opaque request states behind prepare / advance / finish / release.

Model objects never cross the wire; the controller only sees ``state_id``s,
progress rows and artifact metadata.  Output modes: ``file`` (write .npy),
``digest`` (hash only), ``check`` (shape + finiteness only).  Reference:
workers/ditserve/models/base.py:23-131.
"""
from __future__ import annotations

import hashlib
import json
import time
from pathlib import Path

from ..runtime import file_hash

OUTPUT_MODES = ("file", "digest", "check")


def digest(value) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False).encode()).hexdigest()


def positive_int(value, name="steps") -> int:
    if type(value) is not int or value < 1:
        raise ValueError(f"{name} must be a positive integer")
    return value


def artifact(value, path=None, mode="file") -> dict:
    """Persist or fingerprint an output; returns metadata, never the tensor."""
    if mode not in OUTPUT_MODES:
        raise ValueError("output_mode must be file, digest or check")
    started = time.perf_counter()
    import numpy as np
    if hasattr(value, "detach"):
        value = value.detach().float().cpu().numpy()
    arr = np.asarray(value)
    if arr.dtype.kind not in "fiu" or not np.isfinite(arr).all():
        raise ValueError("model output must be a finite numeric array")
    out = {"shape": list(arr.shape), "dtype": str(arr.dtype), "finite": True, "output_mode": mode}
    if mode != "check":
        out["array_sha256"] = hashlib.sha256(np.ascontiguousarray(arr).tobytes()).hexdigest()
    if mode == "file" and path:
        dest = Path(path).resolve()
        if dest.suffix != ".npy":
            raise ValueError("array output path must end in .npy")
        dest.parent.mkdir(parents=True, exist_ok=True)
        with dest.open("xb") as f:
            np.save(f, arr, allow_pickle=False)
        out["path"] = str(dest)
        out["bytes"] = dest.stat().st_size
        out["sha256"] = file_hash(dest)
    out["persistence_ms"] = (time.perf_counter() - started) * 1000
    return out


def transfer_dir(config: dict) -> str:
    """Directory of host-staged continuation packets: the worker config's ``transfer_dir``,
    else ``DITSERVE_TRANSFER_DIR``, else /dev/shm (tmpfs) when present, else /tmp."""
    import os
    return str(config.get("transfer_dir") or os.environ.get("DITSERVE_TRANSFER_DIR")
               or ("/dev/shm" if os.path.isdir("/dev/shm") else "/tmp"))


def progress(step, steps, *, done=None, next_action=None) -> dict:
    done = step >= steps if done is None else bool(done)
    return dict(step=step, steps=steps, done=done, next_action=next_action or ("finish" if done else "advance"))


class Backend:
    operations = ("prepare", "advance", "finish", "release")

    def __init__(self, config: dict):
        self.config = config
        self.states: dict = {}

    def state(self, request):
        key = request.get("state_id", request.get("snapshot_id"))
        if not isinstance(key, str) or key not in self.states:
            raise ValueError("unknown state_id")
        return self.states[key]

    def new_id(self, request) -> str:
        key = request.get("state_id", request.get("spec", {}).get("request_id"))
        if not isinstance(key, str) or not key:
            raise ValueError("prepare requires a nonempty state_id or spec.request_id")
        if key in self.states:
            raise ValueError("duplicate live state_id")
        return key

    def output_path(self, request, suffix=".npy"):
        key = hashlib.sha256(str(request.get("state_id", "batch")).encode()).hexdigest()[:16]
        return request.get("output_path") or str(Path(self.config.get("work_dir", ".")) /
                                                 f"output-{key}-{request['id']}{suffix}")

    def persist(self, value, request, suffix=".npy"):
        return artifact(value, self.output_path(request, suffix), request.get("output_mode", "file"))

    def release(self, request):
        self.state(request)
        del self.states[request["state_id"]]
        return dict(released=request["state_id"])

    def capabilities(self) -> dict:
        return {}

    def close(self):
        for key in list(self.states):
            self.release({"state_id": key})
