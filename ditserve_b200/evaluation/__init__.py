"""Quality metrics, dataset splits and telemetry parsers.

* ``psnr``, ``ssim`` (Gaussian-window SSIM, Wang et al. 2004) on [-1, 1] or [0, 1] video/image
  tensors; ``drift`` = cosine + relative L2 (the cross-parallelism gate: cos >= 0.95, relL2 <= 0.25).
* ``lpips`` needs pretrained AlexNet/VGG weights, which are not available offline; the function
  takes a feature network and raises a clear error without one.
* ``hash_bucket_split`` — deterministic train/val/test assignment by SHA-256 of an item id.
* ``kineto_summary`` — aggregate GPU kernel time by name from a torch.profiler chrome trace.
* ``nsys_gpu_metrics`` — per-device busy time, top kernels, copies and NVTX ranges from an Nsight
  Systems SQLite export.
Submodules: ``vbench`` (generation protocol, video export and the pinned official evaluator),
``datasets`` (VBench / VidProM / DiffusionDB prompt manifests from local files, dev / test roles),
``collectives`` (all-to-all bandwidth microbench of the communication backend).
Reference: workers/ditserve/evaluation/{quality.py:39-125, artifacts.py:186-345, datasets.py,
cuda_profile.py}.
"""
from __future__ import annotations

import hashlib
import json
import math
from collections import defaultdict

import torch
import torch.nn.functional as F


def _unit(x: torch.Tensor, value_range) -> torch.Tensor:
    lo, hi = value_range
    return (x.float() - lo) / (hi - lo)


def psnr(a: torch.Tensor, b: torch.Tensor, value_range=(-1.0, 1.0)) -> float:
    mse = F.mse_loss(_unit(a, value_range), _unit(b, value_range)).item()
    return float("inf") if mse == 0 else 10.0 * math.log10(1.0 / mse)


def _gauss(size=11, sigma=1.5, device=None):
    x = torch.arange(size, dtype=torch.float32, device=device) - size // 2
    g = torch.exp(-x ** 2 / (2 * sigma ** 2))
    g = g / g.sum()
    return g[:, None] * g[None, :]


def ssim(a: torch.Tensor, b: torch.Tensor, value_range=(-1.0, 1.0)) -> float:
    """Mean SSIM over frames/channels; inputs [..., H, W] (video [B, C, T, H, W] allowed)."""
    x = _unit(a, value_range).reshape(-1, 1, *a.shape[-2:])
    y = _unit(b, value_range).reshape(-1, 1, *b.shape[-2:])
    w = _gauss(device=x.device)[None, None]
    pad = w.shape[-1] // 2
    mu_x, mu_y = F.conv2d(x, w, padding=pad), F.conv2d(y, w, padding=pad)
    sxx = F.conv2d(x * x, w, padding=pad) - mu_x ** 2
    syy = F.conv2d(y * y, w, padding=pad) - mu_y ** 2
    sxy = F.conv2d(x * y, w, padding=pad) - mu_x * mu_y
    c1, c2 = 0.01 ** 2, 0.03 ** 2
    s = ((2 * mu_x * mu_y + c1) * (2 * sxy + c2)) / ((mu_x ** 2 + mu_y ** 2 + c1) * (sxx + syy + c2))
    return s.mean().item()


def drift(a: torch.Tensor, b: torch.Tensor) -> dict:
    x, y = a.double().flatten(), b.double().flatten()
    cos = (x @ y / (x.norm() * y.norm()).clamp_min(1e-300)).item()
    rel = ((x - y).norm() / y.norm().clamp_min(1e-300)).item()
    return dict(cos=cos, rel_l2=rel, passes=cos >= 0.95 and rel <= 0.25)


def lpips(a, b, feature_net=None):
    if feature_net is None:
        raise RuntimeError("LPIPS needs pretrained AlexNet/VGG features, which are not available offline")
    fa, fb = feature_net(a), feature_net(b)
    return sum(((F.normalize(x, dim=1) - F.normalize(y, dim=1)) ** 2).mean().item() for x, y in zip(fa, fb))


def hash_bucket_split(ids, fractions=(("train", 0.8), ("val", 0.1), ("test", 0.1)), salt: str = "ditserve"):
    total = sum(f for _, f in fractions)
    out = defaultdict(list)
    for i in ids:
        h = int(hashlib.sha256(f"{salt}:{i}".encode()).hexdigest()[:15], 16) / float(1 << 60)
        acc = 0.0
        for name, f in fractions:
            acc += f / total
            if h < acc:
                out[name].append(i)
                break
        else:
            out[fractions[-1][0]].append(i)
    return dict(out)


def kineto_summary(trace_path: str, top: int = 20) -> list:
    """[{name, calls, total_us, share}] of GPU kernels in a chrome trace (torch.profiler export)."""
    data = json.load(open(trace_path))
    events = data["traceEvents"] if isinstance(data, dict) else data
    agg = defaultdict(lambda: [0, 0.0])
    for ev in events:
        if ev.get("ph") == "X" and ev.get("cat") in ("kernel", "gpu_memcpy", "gpu_memset"):
            a = agg[ev["name"]]
            a[0] += 1
            a[1] += float(ev.get("dur", 0.0))
    tot = sum(v[1] for v in agg.values()) or 1.0
    rows = [dict(name=k, calls=v[0], total_us=round(v[1], 2), share=round(v[1] / tot, 4)) for k, v in agg.items()]
    rows.sort(key=lambda r: -r["total_us"])
    return rows[:top]


def _union_ns(intervals) -> int:
    busy, end = 0, None
    for s, e in sorted(intervals):
        if end is None or s > end:
            busy += e - s
            end = e
        elif e > end:
            busy += e - end
            end = e
    return busy


def nsys_gpu_metrics(sqlite_path: str, top: int = 20) -> dict:
    """GPU metrics from an Nsight Systems SQLite export (``nsys export --type sqlite``).

    Reads the documented export tables: ``CUPTI_ACTIVITY_KIND_KERNEL`` (start, end, deviceId,
    shortName -> ``StringIds``), ``CUPTI_ACTIVITY_KIND_MEMCPY`` (start, end, bytes, copyKind) and,
    when present, ``NVTX_EVENTS`` ranges (start, end, text).  Returns per-device busy time (the
    union of kernel intervals, so concurrent streams are not double counted) over the span from
    the first to the last GPU activity, the top kernels by total time, copy totals per kind and
    NVTX range totals.  Reference: the Nsight Systems metric parser of the reference's evaluation
    tooling (workers/ditserve/evaluation/nsys_metrics.py)."""
    import sqlite3
    con = sqlite3.connect(f"file:{sqlite_path}?mode=ro", uri=True)
    try:
        tables = {r[0] for r in con.execute("SELECT name FROM sqlite_master WHERE type='table'")}
        names = dict(con.execute("SELECT id, value FROM StringIds")) if "StringIds" in tables else {}
        kernels = []
        if "CUPTI_ACTIVITY_KIND_KERNEL" in tables:
            kernels = list(con.execute("SELECT start, end, deviceId, shortName FROM CUPTI_ACTIVITY_KIND_KERNEL"))
        copies = []
        if "CUPTI_ACTIVITY_KIND_MEMCPY" in tables:
            copies = list(con.execute("SELECT start, end, bytes, copyKind FROM CUPTI_ACTIVITY_KIND_MEMCPY"))
        ranges = []
        if "NVTX_EVENTS" in tables:
            ranges = list(con.execute("SELECT start, end, text FROM NVTX_EVENTS WHERE end IS NOT NULL"))
    finally:
        con.close()
    stamps = [t for k in kernels for t in k[:2]] + [t for c in copies for t in c[:2]]
    span_ns = (max(stamps) - min(stamps)) if stamps else 0
    per_dev = defaultdict(list)
    agg = defaultdict(lambda: [0, 0])
    for s, e, dev, name in kernels:
        per_dev[dev].append((s, e))
        a = agg[names.get(name, str(name))]
        a[0] += 1
        a[1] += e - s
    ktot = sum(v[1] for v in agg.values()) or 1
    top_rows = sorted(([k, v[0], v[1]] for k, v in agg.items()), key=lambda r: -r[2])[:top]
    copy_kinds = {1: "HtoD", 2: "DtoH", 8: "DtoD", 10: "PtoP"}
    cagg = defaultdict(lambda: [0, 0, 0])
    for s, e, nbytes, kind in copies:
        c = cagg[copy_kinds.get(kind, str(kind))]
        c[0] += 1
        c[1] += nbytes
        c[2] += e - s
    ragg = defaultdict(lambda: [0, 0])
    for s, e, text in ranges:
        r = ragg[text]
        r[0] += 1
        r[1] += e - s
    return dict(
        span_ms=span_ns / 1e6,
        devices={int(d): dict(busy_ms=_union_ns(iv) / 1e6, utilization=(_union_ns(iv) / span_ns) if span_ns else 0.0,
                               kernels=len(iv)) for d, iv in sorted(per_dev.items())},
        kernels=[dict(name=n, calls=c, total_ms=t / 1e6, share=round(t / ktot, 4)) for n, c, t in top_rows],
        copies={k: dict(count=v[0], bytes=v[1], total_ms=v[2] / 1e6,
                        gbps=(v[1] / v[2]) if v[2] else 0.0) for k, v in cagg.items()},
        nvtx={k: dict(count=v[0], total_ms=v[1] / 1e6) for k, v in ragg.items()},
    )
