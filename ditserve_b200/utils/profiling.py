"""Profiling helpers: per-module CUDA-event timing and Kineto traces of a request.

``ModuleTimer(model)`` brackets every transformer block with CUDA events and reports
per-block device time after a synchronize: it wraps ``model.forward_block(i, ...)`` where the
model drives its blocks that way (Wan), else registers forward hooks on the top-level
children of ``blocks`` / ``transformer_blocks``; ``kineto_trace(fn, path)`` records a torch.profiler trace of ``fn`` with
NVTX-style record_function ranges and returns the aggregated kernel table.  Numbers taken
under a profiler are for shares, never for benchmark values.
Reference: workers/ditserve/models/profiling.py:25-136, wan/profile.py:142-358.
"""
from __future__ import annotations

import time
from collections import defaultdict

import torch

from ..evaluation import kineto_summary


class ModuleTimer:
    def __init__(self, model: torch.nn.Module, prefixes=("blocks.", "transformer_blocks.")):
        self.handles = []
        self.events = defaultdict(list)
        self.cuda = next(model.parameters()).is_cuda
        self.model = model
        if hasattr(model, "forward_block"):
            inner = model.forward_block

            def timed(i, *a, **k):
                name = f"blocks.{i}"
                self._pre(name)(None, None)
                out = inner(i, *a, **k)
                self._post(name)(None, None, None)
                return out
            model.forward_block = timed
            self.handles.append(_Restore(model, "forward_block"))
            return
        for name, mod in model.named_modules():
            if name.count(".") == 1 and name.startswith(prefixes):
                self.handles.append(mod.register_forward_pre_hook(self._pre(name)))
                self.handles.append(mod.register_forward_hook(self._post(name)))

    def _pre(self, name):
        def hook(mod, args):
            if self.cuda:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                self.events[name].append([e, None])
            else:
                self.events[name].append([time.perf_counter(), None])
        return hook

    def _post(self, name):
        def hook(mod, args, out):
            if self.cuda:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                self.events[name][-1][1] = e
            else:
                self.events[name][-1][1] = time.perf_counter()
        return hook

    def report(self) -> dict:
        if self.cuda:
            torch.cuda.synchronize()
        out = {}
        for name, pairs in self.events.items():
            ms = [(b.elapsed_time(e) if self.cuda else (e - b) * 1000) for b, e in pairs if e is not None]
            out[name] = dict(calls=len(ms), total_ms=round(sum(ms), 3))
        return out

    def close(self):
        for h in self.handles:
            h.remove()


class _Restore:
    def __init__(self, obj, attr):
        self.obj, self.attr = obj, attr

    def remove(self):
        self.obj.__dict__.pop(self.attr, None)


def kineto_trace(fn, path: str, label: str = "ditserve_step", top: int = 20):
    from torch.profiler import ProfilerActivity, profile, record_function
    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
    with profile(activities=acts) as prof:
        with record_function(label):
            fn()
    prof.export_chrome_trace(path)
    return kineto_summary(path, top)
