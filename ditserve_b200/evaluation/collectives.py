"""All-to-all bandwidth microbench of the communication backend (NCCL, or Gloo on CPU).

    torchrun --nproc-per-node N -m ditserve_b200.evaluation.collectives [--sizes-mb 16 64 256]

For each message size (bytes each rank sends in total) the Ulysses exchange primitive,
``all_to_all_single``, runs ``warmup`` untimed and ``iterations`` timed rounds; the time of a
round is the max over ranks (CUDA events on the launching stream on GPUs, a wall clock around a
barrier on the CPU).  Reported per size: time, algorithm bandwidth (bytes sent per rank / time)
and bus bandwidth (algbw x (N-1)/N, the share that actually crosses links).  These are the link
figures the planner's cost profile takes for the all-to-all term.
Reference: workers/ditserve/evaluation/collectives.py:27-95.
"""
from __future__ import annotations

import argparse
import json
import os
import time

import torch
import torch.distributed as dist


def _round_ms(fn, device) -> float:
    if device.type == "cuda":
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize(device)
        ms = s.elapsed_time(e)
    else:
        dist.barrier()
        t0 = time.perf_counter()
        fn()
        ms = (time.perf_counter() - t0) * 1e3
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def measure(sizes_mb=(16, 64, 256), iterations: int = 5, warmup: int = 2, device=None, group=None) -> list:
    world = dist.get_world_size(group)
    device = device or (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
                        else torch.device("cpu"))
    out = []
    for mb in sizes_mb:
        n = int(mb * (1 << 20)) // 2
        n -= n % world
        if n <= 0:
            raise ValueError(f"message of {mb} MB is too small for {world} ranks")
        send = torch.randn(n, device=device).to(torch.bfloat16)
        recv = torch.empty_like(send)
        fn = lambda: dist.all_to_all_single(recv, send, group=group)  # noqa: E731
        for _ in range(warmup):
            fn()
        if device.type == "cuda":
            torch.cuda.synchronize(device)
        times = sorted(_round_ms(fn, device) for _ in range(iterations))
        ms = times[len(times) // 2]
        nbytes = n * 2
        algbw = nbytes / (ms * 1e-3) / 1e9
        out.append(dict(size_mb=mb, bytes=nbytes, ms=round(ms, 4), algbw_gbs=round(algbw, 2),
                        busbw_gbs=round(algbw * (world - 1) / world, 2), world=world))
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes-mb", type=float, nargs="+", default=[16, 64, 256])
    ap.add_argument("--iterations", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    args = ap.parse_args(argv)
    from datetime import timedelta
    if torch.cuda.is_available():
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    rows = measure(args.sizes_mb, args.iterations, args.warmup)
    if dist.get_rank() == 0:
        for r in rows:
            print(json.dumps(r))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
