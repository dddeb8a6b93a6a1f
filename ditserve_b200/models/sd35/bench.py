"""SD3.5-Medium step latency on one GPU: single requests and packed continuous batches.

    python -m ditserve_b200.models.sd35.bench [--steps 5] [--json out.json]

Reports device-timed ms per denoising step (both CFG branches, 333 text tokens, random
weights) for 512^2 and 1024^2 alone and for packed mixes, next to the reference's published
A100 figures (SP1 step 61.6 ms at 512^2 and 218.2 ms at 1024^2; packing 512^2+1024^2
444.88 -> 260.09 ms per step).
"""
from __future__ import annotations

import argparse
import json

import torch

from .model import SD35_MEDIUM
from .runtime import SD35Engine

CASES = {
    "512": [(512, 512)],
    "1024": [(1024, 1024)],
    "512+1024": [(512, 512), (1024, 1024)],
    "4x512": [(512, 512)] * 4,
    "8x512": [(512, 512)] * 8,
    "4x1024": [(1024, 1024)] * 4,
    "mixed8": [(512, 512)] * 4 + [(1024, 1024)] * 4,
}
PUBLISHED_A100_MS = {"512": 61.6, "1024": 218.2, "512+1024": 260.09}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--json", default=None)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    eng = SD35Engine(SD35_MEDIUM, device=dev)
    rows = []
    for name, sizes in CASES.items():
        states = [eng.prepare(dict(height=h, width=w, steps=100, seed=i)) for i, (h, w) in enumerate(sizes)]
        for _ in range(2):
            eng.advance_batch(states)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.steps):
            eng.advance_batch(states)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / args.steps
        row = {"case": name, "requests": len(sizes), "ms_per_step": round(ms, 3),
               "ms_per_request_step": round(ms / len(sizes), 3)}
        if name in PUBLISHED_A100_MS:
            row["reference_a100_ms"] = PUBLISHED_A100_MS[name]
        rows.append(row)
        print(json.dumps(row), flush=True)
    if args.json:
        json.dump(rows, open(args.json, "w"), indent=1)


if __name__ == "__main__":
    main()
