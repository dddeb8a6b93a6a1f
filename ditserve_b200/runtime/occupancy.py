"""GPU occupancy probe: foreign compute processes on our GPUs.

Uses NVML through nvidia-ml-py when present, else ``nvidia-smi``; fails closed
to ``unknown`` (the controller tolerates a bounded number of unknown probes).
Reads only — it never changes a GPU setting.  Reference:
workers/ditserve/runtime/worker.py:312-390, runtime/occupancy_nvml.py:33-193.
"""
from __future__ import annotations

import json
import os
import subprocess


def _nvml_probe(indices):
    import pynvml  # nvidia-ml-py
    pynvml.nvmlInit()
    try:
        out = {}
        for i in indices:
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            procs = pynvml.nvmlDeviceGetComputeRunningProcesses(h)
            out[str(i)] = [{"pid": p.pid, "used_bytes": int(p.usedGpuMemory or 0)} for p in procs]
        return out
    finally:
        pynvml.nvmlShutdown()


def _smi_probe(indices):
    res = subprocess.run(["nvidia-smi", "--query-compute-apps=gpu_bus_id,pid,used_memory", "--format=csv,noheader"],
                         capture_output=True, text=True, timeout=10)
    if res.returncode != 0:
        raise RuntimeError(res.stderr.strip())
    bus = subprocess.run(["nvidia-smi", "--query-gpu=index,pci.bus_id", "--format=csv,noheader"],
                         capture_output=True, text=True, timeout=10)
    index_of = {}
    for line in bus.stdout.strip().splitlines():
        i, b = [c.strip() for c in line.split(",")]
        index_of[b] = int(i)
    out = {str(i): [] for i in indices}
    for line in res.stdout.strip().splitlines():
        b, pid, mem = [c.strip() for c in line.split(",")]
        i = index_of.get(b)
        if i in indices:
            out[str(i)].append({"pid": int(pid), "used_mib": mem})
    return out


def _file_probe(path):
    """A recorded process table ({gpu: [{"pid": ...}]}) read from ``path`` — the stand-in for
    NVML in tests of the controller's occupancy guard (no GPU needed)."""
    def probe(indices):
        with open(path) as f:
            table = json.load(f)
        if table == "fail":
            raise RuntimeError("probe failure (recorded)")
        return {str(i): table.get(str(i), []) for i in indices}
    return probe


def occupancy(indices=None, own_pids=(), probe=None) -> dict:
    """{"state": "idle"|"busy"|"unknown", "foreign": {gpu: [procs]}, "source": ...}"""
    indices = list(indices if indices is not None else range(8))
    if probe is None and os.environ.get("DITSERVE_OCCUPANCY_TABLE"):
        probe = _file_probe(os.environ["DITSERVE_OCCUPANCY_TABLE"])
    own = set(own_pids) | {os.getpid()}
    for name, fn in ([("injected", probe)] if probe else [("nvml", _nvml_probe), ("nvidia-smi", _smi_probe)]):
        try:
            procs = fn(indices)
        except Exception as exc:  # noqa: BLE001 - any failure means "unknown"
            last = f"{name}: {exc}"
            continue
        foreign = {g: [p for p in ps if p["pid"] not in own] for g, ps in procs.items()}
        busy = any(foreign.values())
        return {"state": "busy" if busy else "idle", "foreign": foreign, "source": name}
    return {"state": "unknown", "foreign": {}, "source": last if indices else "no gpus"}
