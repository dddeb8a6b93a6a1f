"""Single-process probes of the fused peer-memory kernels across two GPUs.

    python -m ditserve_b200.parallel.peer_probe [--kernel all|qkv_scatter|attention_scatter|
                                                 allgather_rows|cfg_step_peer] [--iters 10]

One process drives GPU 0 and GPU 1 with direct peer access.  Each probe launches one fused
kernel on GPU 0 as rank 0 of a two-member group whose other member's buffers live on GPU 1,
so the kernel's NVLink traffic is real, but no kernel ever waits for another launch: the
store-only kernels (qkv_scatter, attention_scatter, allgather_rows) never wait, and the
partner flag that cfg_step_peer waits for is written by the host before the launch.  That
makes every probe safe to replay under a profiler, one GPU at a time.

Shapes are those of Wan2.1-1.3B 480p (32 760 tokens, 12 x 128 heads) at SP2, the
per-rank share of the ``cfg2sp2`` form:
  * qkv_scatter:       16 380 local tokens; half of the q/k/v heads cross to GPU 1
                       (16 380 x 3 x 768 x 2 B = 75.5 MB);
  * attention_scatter: 6 heads over 32 760 tokens; the rows of GPU 1's tokens are stored
                       into GPU 1's output buffer (16 380 x 768 x 2 B = 25.2 MB);
  * allgather_rows:    16 380 x 64 bf16 rows stored into both members (2.1 MB cross);
  * cfg_step_peer:     the partner's 16 x 21 x 60 x 104 bf16 prediction is read over
                       NVLink (4.2 MB) and combined with the local one into the fp32 latent.
Each line of output gives the CUDA-event time per launch (median of ``--iters``, 3 warm-up
launches) and the bytes that must cross NVLink, which is the roofline of a fused
compute+collective kernel together with its own FLOPs.
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from ..ops._ext import ext, status_word

TOKENS, HEADS, HEAD_DIM = 32760, 12, 128
LATENT = (16, 21, 60, 104)
CFG_CHANNEL = 1


def _heaps(nbytes: int):
    e = ext()
    if torch.cuda.device_count() < 2:
        raise SystemExit("peer_probe needs two visible GPUs")
    for a, b in ((0, 1), (1, 0)):
        if not e.peer_enable(a, b):
            raise SystemExit(f"GPU {a} cannot access GPU {b} directly")
    h0, _ = e.symm_alloc(nbytes, 0)
    h1, _ = e.symm_alloc(nbytes, 1)
    return h0, h1


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize(0)
    ms = []
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize(0)
        ms.append(e0.elapsed_time(e1))
    ms.sort()
    return ms[len(ms) // 2]


def probe_qkv_scatter(iters: int) -> dict:
    e = ext()
    sl = TOKENS // 2
    width = HEADS * HEAD_DIM
    flag = max(65536, int(e.FLAG_BYTES))
    recv = TOKENS * 3 * (width // 2) * 2
    h0, h1 = _heaps(flag + recv + (1 << 20))
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1)
    qkv = torch.randn(sl, 3 * width, device=dev, generator=g).bfloat16()
    w = torch.ones(width, device=dev, dtype=torch.bfloat16)
    ang = torch.rand(TOKENS, HEAD_DIM // 2, device=dev, generator=g)
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    bases = [h0.data_ptr(), h1.data_ptr()]
    torch.cuda.set_device(0)
    ms = _time(lambda: e.qkv_scatter(qkv, w, w, 1e-6, cos, sin, sl, HEADS, HEAD_DIM, 0, bases, int(2e9), flag, 0),
               iters)
    nvl = sl * 3 * (width // 2) * 2
    hbm = sl * 3 * width * 2 + sl * 3 * (width // 2) * 2  # read qkv, write the local half
    return dict(kernel="qkv_scatter", ms=round(ms, 4), nvlink_bytes=nvl, local_hbm_bytes=hbm,
                nvlink_gbs=round(nvl / ms / 1e6, 1), hbm_gbs=round(hbm / ms / 1e6, 1))


def probe_attention_scatter(iters: int) -> dict:
    e = ext()
    hl = HEADS // 2
    w = hl * HEAD_DIM
    flag = max(65536, int(e.FLAG_BYTES))
    o_bytes = (TOKENS // 2) * HEADS * HEAD_DIM * 2
    h0, h1 = _heaps(flag + o_bytes + (1 << 20))
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(2)
    qkv = torch.randn(TOKENS, 3 * w, device=dev, generator=g).bfloat16()
    q, k, v = qkv[:, :w], qkv[:, w:2 * w], qkv[:, 2 * w:]
    st = status_word(dev)
    bases = [h0.data_ptr(), h1.data_ptr()]
    torch.cuda.set_device(0)
    ms = _time(lambda: e.attention_scatter(q, k, v, 1, TOKENS, hl, HEAD_DIM, 1.0 / math.sqrt(HEAD_DIM), 0, bases,
                                           int(2e9), flag, TOKENS // 2, 0, HEADS * HEAD_DIM, st, [], []), iters)
    flops = 4.0 * hl * TOKENS * TOKENS * HEAD_DIM
    nvl = (TOKENS // 2) * w * 2
    return dict(kernel="attention_scatter", ms=round(ms, 4), tflops=round(flops / ms / 1e9, 1), nvlink_bytes=nvl,
                nvlink_gbs=round(nvl / ms / 1e6, 1))


def probe_allgather_rows(iters: int) -> dict:
    e = ext()
    sl, cols = TOKENS // 2, 64
    flag = max(65536, int(e.FLAG_BYTES))
    h0, h1 = _heaps(flag + 2 * sl * cols * 2 + (1 << 20))
    dev = torch.device("cuda", 0)
    y = torch.randn(sl, cols, device=dev).bfloat16()
    bases = [h0.data_ptr(), h1.data_ptr()]
    torch.cuda.set_device(0)
    ms = _time(lambda: e.allgather_rows(y, flag, 0, bases, int(2e9)), iters)
    nvl = sl * cols * 2
    return dict(kernel="allgather_rows", ms=round(ms, 4), nvlink_bytes=nvl, nvlink_gbs=round(nvl / ms / 1e6, 1))


def probe_cfg_step_peer(iters: int) -> dict:
    e = ext()
    n = math.prod(LATENT)
    flag = max(65536, int(e.FLAG_BYTES))
    slot = n * 2
    h0, h1 = _heaps(flag + 2 * slot + (1 << 20))
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(3)
    mine = torch.randn(n, device=dev, generator=g).bfloat16()
    h1[flag:flag + slot].view(torch.bfloat16).copy_(torch.randn(n, device=dev, generator=g).bfloat16())
    sample = torch.randn(n, device=dev, generator=g)
    st = status_word(dev)
    bases = [h0.data_ptr(), h1.data_ptr()]
    epoch = 1
    # the partner's signal (rank 1 -> rank 0) is in place before every launch, so the kernel
    # never waits: flags[channel][peer] of rank 0's heap holds the epoch already
    max_peers = int(e.MAX_PEERS)
    h0[:int(e.FLAG_BYTES)].view(torch.int64)[CFG_CHANNEL * max_peers + 1] = epoch
    torch.cuda.set_device(0)

    def launch():
        e.cfg_step_peer(mine, flag, 0, 5.0, sample, 0.5, False, None, 0.0, 0.0, [], [], 1.0, 0.0, -0.5, [], [],
                        None, None, 0, bases, int(2e9), CFG_CHANNEL, epoch, st, None)
    ms = _time(launch, iters)
    nvl = n * 2
    hbm = n * 2 + 2 * n * 4  # my prediction, the latent read and written
    return dict(kernel="cfg_step_peer", ms=round(ms, 4), nvlink_bytes=nvl, local_hbm_bytes=hbm,
                nvlink_gbs=round(nvl / ms / 1e6, 1))


PROBES = {"qkv_scatter": probe_qkv_scatter, "attention_scatter": probe_attention_scatter,
          "allgather_rows": probe_allgather_rows, "cfg_step_peer": probe_cfg_step_peer}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", default="all", choices=["all", *PROBES])
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args(argv)
    names = list(PROBES) if args.kernel == "all" else [args.kernel]
    for name in names:
        out = PROBES[name](args.iters)
        torch.cuda.synchronize(0)
        from ..ops import check_status
        check_status(torch.device("cuda", 0))
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
