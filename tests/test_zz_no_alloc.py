"""The allocation-free C entry point (ds_fused_qkv_attention_noalloc), called through its
exported C symbol with ctypes.

It is meant for callers that may not allocate GPU memory themselves (an application that
owns all device memory in its own pool, a plugin inside another framework, a serving loop
that must stay out of the driver allocator).  Its output must match the existing
heap-backed path — the qkv_scatter kernel staging q/k/v in a cudaMalloc'd buffer, then the
attention kernel — on two calls in a row, the second smaller than the first (the static
scratch array keeps the previous call's contents, which must not leak into the next
result), and an independent fp32 PyTorch statement of the same math.  This file is collected last
so a failing run has already exercised every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, TOO_LARGE, BAD_ARGUMENT = 0, 1, 2


def _entry():
    from ditserve_b200 import _C
    lib = ctypes.CDLL(_C.__file__)
    fn = lib.ds_fused_qkv_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _existing_path(qkv, wq, wk, eps, cos, sin, batch, seq, heads, hd):
    """The heap-backed entry point: qkv_scatter into a cudaMalloc'd buffer, then attention."""
    from ditserve_b200 import ops
    ext = ops.ext()
    width = heads * hd
    heap, _ = ext.symm_alloc(int(ext.FLAG_BYTES) + batch * seq * 3 * width * 2 + 4096, 0)
    off = 4096 if int(ext.FLAG_BYTES) <= 4096 else int(ext.FLAG_BYTES)
    ext.qkv_scatter(qkv, wq, wk, float(eps), cos, sin, seq, heads, hd, 0, [heap.data_ptr()], int(1e9), off, 0)
    staged = heap[off:off + batch * seq * 3 * width * 2].view(torch.bfloat16).view(batch * seq, 3 * width)
    q, k, v = staged[:, :width], staged[:, width:2 * width], staged[:, 2 * width:]
    out = ops.attention(q.view(batch, seq, width), k.view(batch, seq, width), v.view(batch, seq, width), heads)
    torch.cuda.synchronize()
    return out.reshape(batch * seq, width), heap


def _case(seed, batch, seq, heads, hd, dev):
    g = torch.Generator(device="cpu").manual_seed(seed)
    width = heads * hd
    qkv = torch.randn(batch * seq, 3 * width, generator=g).bfloat16().to(dev)
    wq = (1 + 0.1 * torch.randn(width, generator=g)).bfloat16().to(dev)
    wk = (1 + 0.1 * torch.randn(width, generator=g)).bfloat16().to(dev)
    ang = torch.rand(seq, hd // 2, generator=g) * 5
    return qkv, wq, wk, ang.cos().contiguous().to(dev), ang.sin().contiguous().to(dev)


def _fp32_statement(qkv, wq, wk, eps, cos, sin, batch, seq, heads, hd):
    """Plain fp32 PyTorch: RMS norm across the heads of q and of k, interleaved-pair RoPE,
    softmax attention.  Shares no code with the kernels."""
    width = heads * hd
    x = qkv.float()
    q, k, v = x[:, :width], x[:, width:2 * width], x[:, 2 * width:3 * width]

    def norm(t, w):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * w.float()

    def rope(t):
        pos = torch.arange(t.shape[0], device=t.device) % seq
        c = cos[pos].repeat(1, heads)
        s_ = sin[pos].repeat(1, heads)
        t0, t1 = t[:, 0::2], t[:, 1::2]
        y = torch.empty_like(t)
        y[:, 0::2] = t0 * c - t1 * s_
        y[:, 1::2] = t0 * s_ + t1 * c
        return y

    q, k = rope(norm(q, wq)), rope(norm(k, wk))
    qh = q.view(batch, seq, heads, hd).transpose(1, 2)
    kh = k.view(batch, seq, heads, hd).transpose(1, 2)
    vh = v.view(batch, seq, heads, hd).transpose(1, 2)
    p = torch.softmax((qh @ kh.transpose(-1, -2)) / hd ** 0.5, dim=-1)
    return (p @ vh).transpose(1, 2).reshape(batch * seq, width)


def _call(fn, qkv, wq, wk, eps, cos, sin, batch, seq, heads, hd, dev):
    width = heads * hd
    out = torch.full((batch * seq, width), float("nan"), device=dev, dtype=torch.bfloat16)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = fn(qkv.data_ptr(), qkv.stride(0), batch, seq, heads, hd, wq.data_ptr(), wk.data_ptr(), eps,
            cos.data_ptr(), sin.data_ptr(), out.data_ptr(), out.stride(0), status.data_ptr(), stream)
    torch.cuda.synchronize()
    return rc, out, status


def test_noalloc_entry_matches_heap_path_on_two_calls():
    """Two calls in a row, the second smaller than the first: the second call reads only what
    it staged itself, never the larger first call's leftovers in the shared array."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    fn = _entry()
    heads, hd, eps = 12, 128, 1e-6
    for seed, batch, seq in ((1, 2, 700), (2, 1, 333)):
        qkv, wq, wk, cos, sin = _case(seed, batch, seq, heads, hd, dev)
        ref, _heap = _existing_path(qkv, wq, wk, eps, cos, sin, batch, seq, heads, hd)
        rc, out, status = _call(fn, qkv, wq, wk, eps, cos, sin, batch, seq, heads, hd, dev)
        assert rc == OK
        assert int(status.abs().sum()) == 0
        assert torch.isfinite(out.float()).all()
        torch.testing.assert_close(out.float(), ref.float(), rtol=3e-2, atol=3e-2)


def test_noalloc_entry_matches_fp32_statement():
    """Checked against an independent fp32 statement of norm + RoPE + attention, so a fault
    shared by the staging kernel of both entry points cannot pass unnoticed."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    fn = _entry()
    batch, seq, heads, hd, eps = 2, 300, 12, 128, 1e-6
    qkv, wq, wk, cos, sin = _case(7, batch, seq, heads, hd, dev)
    rc, out, status = _call(fn, qkv, wq, wk, eps, cos, sin, batch, seq, heads, hd, dev)
    assert rc == OK and int(status.abs().sum()) == 0
    ref = _fp32_statement(qkv, wq, wk, eps, cos, sin, batch, seq, heads, hd)
    rel = ((out.float() - ref).norm() / ref.norm()).item()
    assert rel < 2e-2, rel


def test_noalloc_entry_rejects_bad_arguments_before_launching():
    """Misaligned pointers and widths the kernels are not built for come back as
    BAD_ARGUMENT, and nothing is written to the output."""
    dev = torch.device("cuda", 0)
    fn = _entry()
    heads, hd, seq = 12, 128, 64
    width = heads * hd
    qkv, wq, wk, cos, sin = _case(3, 1, seq, heads, hd, dev)
    out = torch.zeros(seq, width, device=dev, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream(dev).cuda_stream
    # qkv shifted by one bf16 element: 2-byte aligned only
    rc = fn(qkv.data_ptr() + 2, qkv.stride(0), 1, seq, heads, hd, wq.data_ptr(), wk.data_ptr(), 1e-6,
            cos.data_ptr(), sin.data_ptr(), out.data_ptr(), out.stride(0), None, stream)
    assert rc == BAD_ARGUMENT
    # 10 heads x 128 = 1280 columns: a multiple of 256 the norm kernel has no instance for
    rc = fn(qkv.data_ptr(), qkv.stride(0), 1, seq, 10, hd, wq.data_ptr(), wk.data_ptr(), 1e-6,
            cos.data_ptr(), sin.data_ptr(), out.data_ptr(), out.stride(0), None, stream)
    assert rc == BAD_ARGUMENT
    torch.cuda.synchronize()
    assert int(out.abs().sum().item()) == 0


def test_noalloc_entry_rejects_problems_beyond_its_array():
    dev = torch.device("cuda", 0)
    fn = _entry()
    heads, hd = 12, 128
    seq = (16 << 20) // (3 * heads * hd * 2) + 1  # one row more than the 16 MiB array holds
    qkv = torch.zeros(seq, 3 * heads * hd, device=dev, dtype=torch.bfloat16)
    w = torch.ones(heads * hd, device=dev, dtype=torch.bfloat16)
    out = torch.zeros(seq, heads * hd, device=dev, dtype=torch.bfloat16)
    rc = fn(qkv.data_ptr(), qkv.stride(0), 1, seq, heads, hd, w.data_ptr(), w.data_ptr(), 1e-6, None, None,
            out.data_ptr(), out.stride(0), None, torch.cuda.current_stream(dev).cuda_stream)
    assert rc == TOO_LARGE
