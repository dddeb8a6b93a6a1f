"""Resident worker process: one backend, JSON-lines protocol v1 over stdin/stdout.

    python -m ditserve_b200.runtime.worker --backend mock|wan|sd35|results|environment [--config JSON]

* Strict framing: one reply per input line; malformed lines get an error reply
  (id null) instead of killing the worker.  NaN/Infinity are rejected.
* stdout is re-routed to stderr at start-up so native libraries or stray prints
  cannot corrupt the framing; replies go to a private duplicate of the original
  stdout.
* The backend is constructed lazily on the first model op (load time reported);
  ``release`` of an unknown state is an error, releasing twice is idempotent.
* Host ops served without a backend: hello (capabilities), occupancy, memory,
  mps_control, shutdown.
Reference: workers/ditserve/runtime/worker.py:108-443.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

from . import PROTOCOL_VERSION
from . import protocol

BACKENDS = {
    "mock": "ditserve_b200.models.mock:MockBackend",
    "wan": "ditserve_b200.models.wan.backend:WanBackend",
    "sd35": "ditserve_b200.models.sd35.backend:SD35Backend",
    "results": "ditserve_b200.results:ResultsBackend",
    "environment": "ditserve_b200.runtime.environment:EnvironmentBackend",
}


def _load_class(path: str):
    mod, _, cls = path.partition(":")
    module = __import__(mod, fromlist=[cls])
    return getattr(module, cls)


class Worker:
    def __init__(self, backend: str, config: dict | None = None):
        if backend not in BACKENDS:
            raise ValueError(f"unknown backend {backend!r}")
        self.backend_name = backend
        self.config = config or {}
        self.backend = None
        self.load_ms = None
        self.released: set = set()
        self.started = time.time()

    def _backend(self):
        if self.backend is None:
            t0 = time.perf_counter()
            self.backend = _load_class(BACKENDS[self.backend_name])(self.config)
            self.load_ms = (time.perf_counter() - t0) * 1000
        return self.backend

    def hello(self, request) -> dict:
        caps = dict(protocol=PROTOCOL_VERSION, backend=self.backend_name, pid=os.getpid(),
                    engine="ditserve_b200", qualification="fixture_only" if self.backend_name == "mock" else "model")
        if self.backend_name in ("mock", "wan", "sd35"):
            b = self._backend()
            caps["operations"] = list(b.operations)
            caps.update(b.capabilities())
            caps["load_ms"] = self.load_ms
        return caps

    def dispatch(self, request: dict):
        op = protocol.operation(request)
        if op == "hello":
            return self.hello(request)
        if op == "occupancy":
            from .occupancy import occupancy
            return occupancy(request.get("gpus"), request.get("own_pids", ()))
        if op == "memory":
            return process_memory()
        if op == "mps_control":
            from .green_context import mps_control
            return mps_control(request, allowed=bool(self.config.get("allow_mps_control", False)))
        if op == "shutdown":
            if self.backend is not None and hasattr(self.backend, "close"):
                self.backend.close()
            return dict(shutdown=True)
        backend = self._backend()
        if op not in backend.operations:
            raise ValueError(f"backend {self.backend_name} has no op {op!r}")
        if op == "release":
            sid = request.get("state_id")
            if sid in self.released and sid not in backend.states:
                return dict(released=sid, idempotent=True)
            out = backend.release(request)
            self.released.add(sid)
            return out
        t0 = time.perf_counter()
        out = getattr(backend, op)(request)
        if isinstance(out, dict):
            out.setdefault("op_ms", (time.perf_counter() - t0) * 1000)
        return out


def process_memory() -> dict:
    out = {"rss_bytes": None}
    try:
        with open("/proc/self/statm") as f:
            out["rss_bytes"] = int(f.read().split()[1]) * os.sysconf("SC_PAGE_SIZE")
    except OSError:
        pass
    if "torch" in sys.modules:
        import torch
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            out["cuda_allocated"] = torch.cuda.memory_allocated()
            out["cuda_reserved"] = torch.cuda.memory_reserved()
    return out


def serve(worker: Worker, incoming, outgoing) -> int:
    for line in incoming:
        if not line.strip():
            continue
        rid = None
        try:
            req = protocol.loads(line)
            rid = req.get("id") if isinstance(req, dict) else None
            result = worker.dispatch(req)
            reply = protocol.ok(rid, result)
            text = protocol.dumps(reply)
        except Exception as exc:  # noqa: BLE001 - every failure becomes a reply
            text = protocol.dumps(protocol.error(rid, exc))
        outgoing.write(text + "\n")
        outgoing.flush()
        if isinstance(req, dict) and req.get("op") == "shutdown" and '"ok":true' in text:
            return 0
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--backend", required=True, choices=sorted(BACKENDS))
    ap.add_argument("--config", default="{}")
    args = ap.parse_args(argv)
    config = json.loads(args.config)
    # keep the protocol stream private: everything else printed goes to stderr
    proto_fd = os.dup(1)
    os.dup2(2, 1)
    out = os.fdopen(proto_fd, "w", buffering=1)
    sys.stdout = sys.stderr
    worker = Worker(args.backend, config)
    try:
        return serve(worker, sys.stdin, out)
    finally:
        if worker.backend is not None and hasattr(worker.backend, "close"):
            try:
                worker.backend.close()
            except Exception:  # noqa: BLE001
                pass


if __name__ == "__main__":
    sys.exit(main())
