"""SM partitioning between co-located workers (video / image roles on one GPU).

* ``partition_sms(total, weights, granularity)`` — split a GPU's SMs into per-role
  groups that respect the driver's minimum group size / alignment (host math only).
* ``GreenPool`` — CUDA Green Contexts through cuda-python's driver bindings: split
  the device's SM resource by count, create one green context per role and a
  stream in each, exposed to torch as ``torch.cuda.ExternalStream``.  A green
  context is a per-process resource view; it changes no device setting.
* ``mps_control`` — start/stop/query the MPS control daemon with a verified
  ``quit``.  The daemon is shared by every process of the machine, so this is
  OFF unless the worker config sets ``allow_mps_control`` (it is never used by the
  tests or the benchmark on the shared pool; its tests drive a fake binary).
Reference: workers/ditserve/runtime/green_context.py:34-269, worker.py:121-158.
"""
from __future__ import annotations

import os
import shutil
import subprocess


def partition_sms(total: int, weights, granularity: int = 8, minimum: int = 8) -> list[int]:
    """Split ``total`` SMs in proportion to ``weights``; every share a multiple of
    ``granularity`` and at least ``minimum``; the shares sum to at most ``total``."""
    if total <= 0 or granularity <= 0:
        raise ValueError("total and granularity must be positive")
    w = [float(x) for x in weights]
    if not w or any(x <= 0 for x in w):
        raise ValueError("weights must be positive")
    n = len(w)
    usable = (total // granularity) * granularity
    if n * max(minimum, granularity) > usable:
        raise ValueError(f"{n} groups of >= {minimum} SMs do not fit in {usable} usable SMs")
    units = usable // granularity
    min_units = -(-max(minimum, granularity) // granularity)
    s = sum(w)
    raw = [u * units / s for u in w]
    shares = [max(min_units, int(r)) for r in raw]
    # largest-remainder fill / trim so the units sum exactly to `units`
    while sum(shares) > units:
        i = max(range(n), key=lambda k: (shares[k] - raw[k], shares[k]))
        if shares[i] <= min_units:
            raise ValueError("cannot satisfy the minimum share")
        shares[i] -= 1
    while sum(shares) < units:
        i = max(range(n), key=lambda k: raw[k] - shares[k])
        shares[i] += 1
    return [u * granularity for u in shares]


class GreenPool:
    """Green contexts on one device with SM shares per role (requires CUDA >= 12.4 driver APIs)."""

    def __init__(self, device: int, shares: dict):
        from cuda.bindings import driver as cu  # cuda-python
        import torch
        self.cu = cu
        torch.cuda.init()
        (err,) = cu.cuInit(0)
        self._check(err, "cuInit")
        err, dev = cu.cuDeviceGet(device)
        self._check(err, "cuDeviceGet")
        err, res = cu.cuDeviceGetDevResource(dev, cu.CUdevResourceType.CU_DEV_RESOURCE_TYPE_SM)
        self._check(err, "cuDeviceGetDevResource")
        self.total_sms = res.sm.smCount
        self.roles = list(shares)
        self.streams = {}
        self.contexts = {}
        self.sm_counts = {}
        remaining = res
        for i, role in enumerate(self.roles):
            count = int(shares[role])
            if i == len(self.roles) - 1 and count >= remaining.sm.smCount:
                # the last role takes what is left as it is: a split must come in the driver's
                # SM granularity (8 on this part), which the remainder need not be
                part, rest = remaining, None
            else:
                err, groups, n, rest = cu.cuDevSmResourceSplitByCount(1, remaining, 0, count)
                self._check(err, f"cuDevSmResourceSplitByCount ({role}: {count} of {remaining.sm.smCount} SMs)")
                part = groups[0] if isinstance(groups, (list, tuple)) else groups
            self.sm_counts[role] = int(part.sm.smCount)
            err, desc = cu.cuDevResourceGenerateDesc([part], 1)
            self._check(err, "cuDevResourceGenerateDesc")
            err, gctx = cu.cuGreenCtxCreate(desc, dev, cu.CUgreenCtxCreate_flags.CU_GREEN_CTX_DEFAULT_STREAM)
            self._check(err, "cuGreenCtxCreate")
            err, stream = cu.cuGreenCtxStreamCreate(gctx, cu.CUstream_flags.CU_STREAM_NON_BLOCKING, 0)
            self._check(err, "cuGreenCtxStreamCreate")
            self.contexts[role] = gctx
            self.streams[role] = torch.cuda.ExternalStream(int(stream), device=torch.device("cuda", device))
            remaining = rest

    def _check(self, err, what):
        if int(err) != 0:
            raise RuntimeError(f"{what} failed with CUresult {int(err)}")

    def stream(self, role: str):
        return self.streams[role]

    def status(self) -> dict:
        return dict(total_sms=self.total_sms, roles=self.roles, sm_counts=dict(self.sm_counts))

    def close(self):
        for gctx in self.contexts.values():
            self.cu.cuGreenCtxDestroy(gctx)
        self.contexts.clear()


def mps_control(request: dict, binary: str | None = None, allowed: bool = False) -> dict:
    """{action: status|quit}.  Refused unless ``allowed`` (worker config allow_mps_control)."""
    action = request.get("action", "status")
    exe = binary or request.get("binary") or shutil.which("nvidia-cuda-mps-control")
    if action == "status":
        return dict(available=exe is not None, pipe_dir=os.environ.get("CUDA_MPS_PIPE_DIRECTORY", "/tmp/nvidia-mps"))
    if not allowed:
        raise PermissionError("MPS control is disabled (the daemon is shared by every process on the machine)")
    if exe is None:
        raise FileNotFoundError("nvidia-cuda-mps-control not found")
    if action == "quit":
        r = subprocess.run([exe], input="quit\n", capture_output=True, text=True, timeout=30)
        if r.returncode != 0:
            raise RuntimeError(f"mps quit failed: {r.stderr.strip()}")
        # verify: a second query must find no daemon
        chk = subprocess.run([exe], input="get_server_list\n", capture_output=True, text=True, timeout=30)
        return dict(quit=True, verified=chk.returncode != 0 or not chk.stdout.strip())
    raise ValueError(f"unknown MPS action {action!r}")
