"""Loader for the sm_100a extension and the per-device kernel status word.

CUDA tensors always go through the hand-written kernels in ``ditserve_b200._C``;
if the extension is missing on a GPU machine every op raises instead of
silently falling back to PyTorch.  CPU tensors use the reference math in each
op module (that path exists for the CPU/Gloo contract tests).
"""
from __future__ import annotations

import threading

import torch

_lock = threading.Lock()
_ext = None
_ext_error: Exception | None = None
_status: dict[int, torch.Tensor] = {}


def ext():
    """Return the compiled extension module, raising if it was not built."""
    global _ext, _ext_error
    if _ext is not None:
        return _ext
    with _lock:
        if _ext is None and _ext_error is None:
            try:
                from .. import _C  # type: ignore[attr-defined]
                _ext = _C
            except Exception as exc:  # pragma: no cover - depends on the build
                _ext_error = exc
    if _ext is None:
        raise RuntimeError(
            "ditserve_b200._C is not built (run `python setup.py build_ext --inplace`); "
            f"CUDA ops have no fallback: {_ext_error!r}")
    return _ext


_launches: dict[str, int] = {}
_timer: "KernelTimer | None" = None


class KernelTimer:
    """Device time per extension entry point, from CUDA events on the launching stream.

    While active (``with KernelTimer() as kt:``) every ``kernel(name)`` call is bracketed by
    two events on the current stream; ``totals_ms()`` synchronises and sums the elapsed
    time per entry-point name.  The events add a few microseconds of host work per launch,
    so the timer is for breakdowns of an untimed step, never for the timed region.
    """

    def __init__(self):
        self.records: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    def __enter__(self):
        global _timer
        self._prev, _timer = _timer, self
        return self

    def __exit__(self, *exc):
        global _timer
        _timer = self._prev
        return False

    def wrap(self, name: str, fn):
        def timed(*args, **kwargs):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out = fn(*args, **kwargs)
            e1.record()
            self.records.append((name, e0, e1))
            return out
        return timed

    def totals_ms(self) -> dict[str, float]:
        torch.cuda.synchronize()
        out: dict[str, float] = {}
        for name, e0, e1 in self.records:
            out[name] = out.get(name, 0.0) + e0.elapsed_time(e1)
        return out


def kernel(name: str):
    """The bound extension entry point ``name``; counts one launch per call (and times it
    while a ``KernelTimer`` is active)."""
    fn = getattr(ext(), name)
    _launches[name] = _launches.get(name, 0) + 1
    if _timer is not None:
        return _timer.wrap(name, fn)
    return fn


def launch_counts(reset: bool = False) -> dict[str, int]:
    """Kernel launches issued through this package since the last reset (host-side count)."""
    out = dict(_launches)
    if reset:
        _launches.clear()
    return out


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def status_word(device: torch.device) -> torch.Tensor:
    """Device int32[2] (code, site) that kernels write when a bounded wait expires."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _status.get(idx)
    if buf is None:
        with _lock:
            buf = _status.get(idx)
            if buf is None:
                buf = torch.zeros(2, dtype=torch.int32, device=torch.device("cuda", idx))
                _status[idx] = buf
    return buf


class KernelTimeout(RuntimeError):
    """A device-side wait gave up; the kernel returned early with an error status."""


STATUS_NAMES = {1: "mbarrier wait timed out", 2: "peer flag wait timed out", 3: "device argument check failed"}


def check_status(device: torch.device | None = None, reset: bool = True) -> None:
    """Synchronise and raise if any kernel on ``device`` reported an error status."""
    devices = [device] if device is not None else [torch.device("cuda", i) for i in list(_status)]
    for dev in devices:
        buf = status_word(dev)
        code, site = (int(v) for v in buf.cpu().tolist())
        if code != 0:
            if reset:
                buf.zero_()
            raise KernelTimeout(f"{STATUS_NAMES.get(code, 'error')} (code {code}, site {site}) on {dev}")


def use_kernels(*tensors: torch.Tensor) -> bool:
    """True when the tensors live on a CUDA device (the kernel path is mandatory there)."""
    return any(t is not None and t.is_cuda for t in tensors)
