"""The allocation-free C entry point (ds_fused_qkv_attention_noalloc), called through its
exported C symbol with ctypes.

It is meant for callers that may not allocate GPU memory themselves (an application that
owns all device memory in its own pool, a plugin inside another framework, a serving loop
that must stay out of the driver allocator).  Its output must match the existing
heap-backed path — the qkv_scatter kernel staging q/k/v in a cudaMalloc'd buffer, then the
attention kernel — on two calls in a row (the static scratch array keeps the previous
call's contents, which must not leak into the next result).  This file is collected last
so a failing run has already exercised every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, TOO_LARGE = 0, 1


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


def test_noalloc_entry_matches_heap_path_on_two_calls():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    fn = _entry()
    batch, seq, heads, hd, eps = 2, 700, 12, 128, 1e-6
    width = heads * hd
    stream = torch.cuda.current_stream(dev).cuda_stream
    for seed in (1, 2):  # two calls in a row: the second must not see the first call's data
        qkv, wq, wk, cos, sin = _case(seed, batch, seq, heads, hd, dev)
        ref, _heap = _existing_path(qkv, wq, wk, eps, cos, sin, batch, seq, heads, hd)
        out = torch.full((batch * seq, width), float("nan"), device=dev, dtype=torch.bfloat16)
        status = torch.zeros(2, dtype=torch.int32, device=dev)
        rc = fn(qkv.data_ptr(), qkv.stride(0), batch, seq, heads, hd, wq.data_ptr(), wk.data_ptr(), eps,
                cos.data_ptr(), sin.data_ptr(), out.data_ptr(), out.stride(0), status.data_ptr(), stream)
        assert rc == OK
        torch.cuda.synchronize()
        assert int(status.abs().sum()) == 0
        assert torch.isfinite(out.float()).all()
        torch.testing.assert_close(out.float(), ref.float(), rtol=3e-2, atol=3e-2)


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
