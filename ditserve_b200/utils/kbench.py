"""Isolated kernel timing against the measured roofline (CUDA events, warm-up, L2 flush).

    python -m ditserve_b200.utils.kbench [--json out.json]

Times the hot ops of one Wan2.1-1.3B 480p block at the bench shapes (M = 2 x 32 760
tokens) on our sm_100a kernels and, for context, on cuBLAS (torch.matmul) and
FlashAttention-2 / torch SDPA when present.  Fractions use MEASURED_PEAKS.json when
it exists (bf16_tflops burst, hbm_gbs), else the pool's fallback figures.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from .. import ops

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["bf16_tflops"], d["hbm_gbs"], "measured"
    return 1590.0, 6650.0, "fallback"


def timeit(fn, iters=10, warmup=3, flush=None):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", default=None)
    ap.add_argument("--tokens", type=int, default=32760)
    ap.add_argument("--batch", type=int, default=2)
    ap.add_argument("--heads", type=int, default=12, help="attention heads of --only attention (the per-GPU heads of a form)")
    ap.add_argument("--only", default=None, help="'fused': only the peer-memory kernels on a one-member group; 'attention': self-attention only; "
                         "'memory': the per-token norm kernels and qkv_scatter; 'cross': cross-attention (512 keys) only; 'trace': SM-clock timeline of one self-attention CTA")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    tflops_peak, hbm_peak, src = peaks()
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev, dtype=torch.float32)  # 256 MB > L2
    S, B, D, F, H = args.tokens, args.batch, 1536, 8960, 12
    M = S * B
    res = {"peaks": {"bf16_tflops": tflops_peak, "hbm_gbs": hbm_peak, "source": src}, "rows": []}

    def row(name, ms, flops=None, bytes_=None, **kw):
        r = {"op": name, "ms": round(ms, 4)}
        if flops:
            r["tflops"] = round(flops / ms / 1e9, 1)
            r["frac_of_" + src] = round(flops / ms / 1e9 / tflops_peak, 3)
        if bytes_:
            r["gbs"] = round(bytes_ / ms / 1e6, 1)
            r["hbm_frac_of_" + src] = round(bytes_ / ms / 1e6 / hbm_peak, 3)
        r.update(kw)
        res["rows"].append(r)
        print(json.dumps(r))

    torch.manual_seed(0)
    if args.only == "attention":
        H = args.heads
        D = H * 128
        qkv = torch.randn(M, 3 * D, device=dev).bfloat16()
        q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
        o = torch.empty(M, D, device=dev, dtype=torch.bfloat16)
        ms = timeit(lambda: ops.attention(q.view(B, S, D), k.view(B, S, D), v.view(B, S, D), H, out=o), iters=5)
        ops.check_status(dev)  # a kernel whose bounded waits ran out raises here instead of printing a time
        row("self_attention", ms, flops=4.0 * B * H * S * S * 128, impl="ours", shape=[B, S, H, 128])
        if args.json:
            json.dump(res, open(args.json, "w"), indent=1)
        return
    if args.only == "trace":
        attention_timeline(dev, S, B, D, H)
        return
    if args.only == "cross":
        q = torch.randn(M, D, device=dev).bfloat16()
        kv = torch.randn(B * 512, 2 * D, device=dev).bfloat16()
        o = torch.empty(M, D, device=dev, dtype=torch.bfloat16)
        ms = timeit(lambda: ops.attention(q.view(B, S, D), kv[:, :D].view(B, 512, D), kv[:, D:].view(B, 512, D), H,
                                          out=o), iters=5)
        ops.check_status(dev)
        row("cross_attention", ms, flops=4.0 * B * H * S * 512 * 128, impl="ours")
        if args.json:
            json.dump(res, open(args.json, "w"), indent=1)
        return
    if args.only == "memory":
        memory_rows(row, timeit, dev, S, B, D, H, flush)
        fused_rows(row, timeit, dev, S, B, D, H, flush, only=("qkv_scatter",))
        if args.json:
            json.dump(res, open(args.json, "w"), indent=1)
        return
    if args.only == "fused":
        fused_rows(row, timeit, dev, S, B, D, H, flush)
        if args.json:
            json.dump(res, open(args.json, "w"), indent=1)
        return
    x = torch.randn(M, D, device=dev).bfloat16()
    for name, N, K, kw in [("qkv_proj", 3 * D, D, {}), ("out_proj_plain", D, D, {}), ("out_proj_gated", D, D, {"gate": True}),
                           ("ffn_up_gelu", F, D, {"act": "gelu"}), ("ffn_down_gated", D, F, {"gate": True})]:
        a = torch.randn(M, K, device=dev).bfloat16()
        w = (torch.randn(N, K, device=dev) / math.sqrt(K)).bfloat16()
        b = torch.randn(N, device=dev).bfloat16()
        extra = {}
        if kw.get("act"):
            extra["act"] = "gelu"
        if kw.get("gate"):
            extra["residual"] = torch.randn(M, N, device=dev).bfloat16()
            extra["gate"] = torch.randn(B, N, device=dev)
            extra["rows_per_batch"] = S
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        ms = timeit(lambda: ops.linear(a, w, b, out=out, **extra), flush=flush)
        row(name, ms, flops=2.0 * M * N * K, impl="ours", shape=[M, N, K])
        ms_cb = timeit(lambda: torch.matmul(a, w.t()), flush=flush)
        row(name + "_cublas_plain", ms_cb, flops=2.0 * M * N * K, impl="cublas", shape=[M, N, K])
        del a, w, out, extra
    # attention
    qkv = torch.randn(M, 3 * D, device=dev).bfloat16()
    q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
    o = torch.empty(M, D, device=dev, dtype=torch.bfloat16)
    fl = 4.0 * B * H * S * S * 128
    ms = timeit(lambda: ops.attention(q.view(B, S, D), k.view(B, S, D), v.view(B, S, D), H, out=o), iters=5)
    row("self_attention", ms, flops=fl, impl="ours", shape=[B, S, H, 128])
    qh = q.reshape(B, S, H, 128)
    kh = k.reshape(B, S, H, 128)
    vh = v.reshape(B, S, H, 128)
    try:
        from flash_attn import flash_attn_func
        qc, kc, vc = qh.contiguous(), kh.contiguous(), vh.contiguous()
        ms = timeit(lambda: flash_attn_func(qc, kc, vc), iters=5)
        row("self_attention_fa2", ms, flops=fl, impl="flash_attn 2 (library)")
    except Exception as exc:  # pragma: no cover
        print("fa2 unavailable", exc)
    try:
        from torch.nn.attention import SDPBackend, sdpa_kernel
        qt, kt, vt = (t.transpose(1, 2).contiguous() for t in (qh, kh, vh))
        with sdpa_kernel(SDPBackend.FLASH_ATTENTION):
            ms = timeit(lambda: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt), iters=5)
        row("self_attention_sdpa_flash", ms, flops=fl, impl="torch SDPA flash (reference path)")
    except Exception as exc:  # pragma: no cover
        print("sdpa flash unavailable", exc)
    # cross attention against 512 text tokens
    kv = torch.randn(B * 512, 2 * D, device=dev).bfloat16()
    ms = timeit(lambda: ops.attention(q.view(B, S, D), kv[:, :D].view(B, 512, D), kv[:, D:].view(B, 512, D), H), iters=5)
    row("cross_attention", ms, flops=4.0 * B * H * S * 512 * 128, impl="ours")
    memory_rows(row, timeit, dev, S, B, D, H, flush)
    fused_rows(row, timeit, dev, S, B, D, H, flush)
    ops.check_status(dev)
    if args.json:
        json.dump(res, open(args.json, "w"), indent=1)


def attention_timeline(dev, S, B, D, H):
    """SM-clock timeline of one CTA of the self-attention kernel (middle of the grid): per key
    tile, when the MMA warp got V and each P, issued the next S, and when row 0 of each softmax
    warpgroup saw S, had it loaded, had the max, finished the exponentials and handed P over."""
    from ..ops._ext import ext, status_word
    M = S * B
    qkv = torch.randn(M, 3 * D, device=dev).bfloat16()
    q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
    o = torch.empty(M, D, device=dev, dtype=torch.bfloat16)
    tr = torch.zeros(32 * 24, dtype=torch.int64, device=dev)
    for _ in range(3):  # warm clocks and caches; the last launch's stamps are kept
        tr.zero_()
        ext().attention_trace(q, k, v, o, B, S, H, D // H, 1.0 / math.sqrt(D // H), status_word(dev), tr)
    torch.cuda.synchronize()
    ops.check_status(dev)
    t = tr.view(32, 24).cpu()
    t0 = int(t[0, 0])
    names = ["vfull", "pvA_issued", "sA_next_issued", "pvB_issued", "sB_next_issued",
             "A_sfull", "A_loaded", "A_max", "A_exp", "A_arrive", "B_sfull", "B_loaded", "B_max", "B_exp", "B_arrive",
             "A_arrive_w1", "A_arrive_w2", "A_arrive_w3", "mma_pA0_seen", "mma_pA1_seen"]
    for j in range(32):
        print(json.dumps({"tile": j, **{n: int(t[j, e]) - t0 if int(t[j, e]) else None for e, n in enumerate(names)}}))
    per = (int(t[24, 0]) - int(t[8, 0])) / 16
    a_soft = sum(int(t[j, 8]) - int(t[j, 5]) for j in range(8, 24)) / 16
    b_soft = sum(int(t[j, 13]) - int(t[j, 10]) for j in range(8, 24)) / 16
    a_ld = sum(int(t[j, 6]) - int(t[j, 5]) for j in range(8, 24)) / 16
    print(json.dumps({"cycles_per_tile": per, "A_sfull_to_exp_done": a_soft, "B_sfull_to_exp_done": b_soft,
                      "A_tmem_load": a_ld, "cta_cycles": int(t[0, 23]) - t0 if int(t[0, 23]) else None}))


def memory_rows(row, timeit, dev, S, B, D, H, flush):
    """The memory-bound per-token kernels of a block: adaLN modulate, q/k RMS norm + RoPE."""
    M = S * B
    x = torch.randn(M, D, device=dev).bfloat16()
    mod = torch.randn(B, 6, D, device=dev)
    y = torch.empty_like(x)
    ms = timeit(lambda: ops.layernorm_modulate(x, scale=mod[:, 1], shift=mod[:, 0], rows_per_batch=S, out=y), flush=flush)
    row("layernorm_modulate", ms, bytes_=2 * M * D * 2, impl="ours")
    qkv = torch.randn(M, 3 * D, device=dev).bfloat16()
    w = torch.ones(D, device=dev).bfloat16()
    ang = torch.rand(S, 64, device=dev)
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    ms = timeit(lambda: ops.rmsnorm_rope_(qkv[:, :D], w, cos=cos, sin=sin, rows_per_batch=S), flush=flush)
    row("rmsnorm_rope_q", ms, bytes_=2 * M * D * 2, impl="ours")
    ms = timeit(lambda: ops.rmsnorm_rope_qk_(qkv, w, w, cos=cos, sin=sin, rows_per_batch=S), flush=flush)
    row("rmsnorm_rope_qk", ms, bytes_=2 * M * 2 * D * 2, impl="ours (q and k in one launch)")


def fused_rows(row, timeit, dev, S, B, D, H, flush, only=None):
    """Peer-memory kernels on a one-member group (this GPU's own heap): the stores stay local,
    so these rows measure each kernel's compute and HBM side; NVLink timing comes from the
    multi-GPU selftests."""
    from ..ops._ext import ext, status_word
    M, hd = S * B, 128
    heap, _ = ext().symm_alloc(int(ext().FLAG_BYTES) + 4 * M * 3 * D * 2 + (64 << 20), 0)
    base = [heap.data_ptr()]
    recv_off = 1 << 20
    o_off = recv_off + ((M * 3 * D * 2 + 4095) // 4096) * 4096
    st = status_word(dev)
    tmo = int(5e9)
    qkv = torch.randn(M, 3 * D, device=dev).bfloat16()
    wq = torch.ones(D, device=dev).bfloat16()
    wk = torch.ones(D, device=dev).bfloat16()
    ang = torch.rand(S, hd // 2, device=dev)
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    ms = timeit(lambda: ext().qkv_scatter(qkv, wq, wk, 1e-6, cos, sin, S, H, hd, 0, base, tmo, recv_off, 0),
                flush=flush)
    row("qkv_scatter_norm_rope_a2a", ms, bytes_=2 * M * 3 * D * 2, impl="ours (group of 1)")
    if only is not None and "attention" not in only:
        del heap
        return
    recv = heap[recv_off:recv_off + M * 3 * D * 2].view(torch.bfloat16).view(M, 3 * D)
    q, k, v = recv[:, :D], recv[:, D:2 * D], recv[:, 2 * D:]
    fl = 4.0 * B * H * S * S * hd
    ms = timeit(lambda: ext().attention_scatter(q, k, v, B, S, H, hd, 1.0 / math.sqrt(hd), 0, base, tmo, o_off, S, 0,
                                                D, st, [], []), iters=5)
    row("attention_peer_store_epilogue", ms, flops=fl, impl="ours (group of 1)")
    y = torch.randn(M, 64, device=dev).bfloat16()
    ms = timeit(lambda: ext().allgather_rows(y, o_off, 0, base, tmo), flush=flush)
    row("allgather_rows", ms, bytes_=2 * M * 64 * 2, impl="ours (group of 1)")
    big = torch.randn(32 << 20, device=dev)  # 128 MB
    ms = timeit(lambda: ext().put_peers(big, 1, recv_off, 0, base, tmo), flush=flush)
    row("put_peers_128MB", ms, bytes_=2 * big.numel() * 4, impl="ours (group of 1)")
    out = torch.zeros(1, dtype=torch.int32, device=dev)
    ms = timeit(lambda: ext().group_flag(0, base, tmo, 5, 0, 0, out, st), iters=20)
    row("group_flag_launch", ms, impl="ours (group of 1: launch + signal cost only)")
    del heap


if __name__ == "__main__":
    main()
