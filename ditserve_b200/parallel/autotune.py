"""Collective-path selection per (form, tokens per rank) from measured timings.

The fused peer-memory plans and the NCCL plans of a layout compute the same result; which
is faster depends on the form and on how much data crosses NVLink per step (tokens per SP
rank).  ``selftest`` measures both on a layout and ``record`` appends the measurement to a
JSON table; ``choose`` returns the path with the lower measured step time for the nearest
measured token count of that form, or the default ("fused") when the form was never
measured.  Reference: workers/gfc/autotune.py (per (collective, group size, slice bytes)
path selection from a JSON table).
"""
from __future__ import annotations

import json
import math
import os
from pathlib import Path

DEFAULT_TABLE = Path(__file__).resolve().parents[2] / "configs" / "profiles" / "collectives.json"


def load(path=None) -> list:
    p = Path(path or os.environ.get("DITSERVE_COLLECTIVES_TABLE", DEFAULT_TABLE))
    if not p.exists():
        return []
    return json.loads(p.read_text()).get("entries", [])


def record(path, form: str, tokens_per_rank: int, nccl_ms: float, fused_ms: float, bitwise: bool, **meta):
    p = Path(path)
    table = json.loads(p.read_text()) if p.exists() else {"version": "ditserve-b200.collectives.v1", "entries": []}
    entry = dict(form=form, tokens_per_rank=int(tokens_per_rank), nccl_ms=float(nccl_ms), fused_ms=float(fused_ms),
                 bitwise=bool(bitwise), **meta)
    table["entries"] = [e for e in table["entries"]
                        if not (e["form"] == form and e["tokens_per_rank"] == entry["tokens_per_rank"])] + [entry]
    p.write_text(json.dumps(table, indent=1, sort_keys=True))
    return entry


def choose(form: str, tokens_per_rank: int, entries=None, default: str = "fused") -> str:
    entries = load() if entries is None else entries
    same = [e for e in entries if e["form"] == form]
    if not same:
        return default
    near = min(same, key=lambda e: abs(math.log(max(1, e["tokens_per_rank"])) - math.log(max(1, tokens_per_rank))))
    return "fused" if near["fused_ms"] <= near["nccl_ms"] else "nccl"
