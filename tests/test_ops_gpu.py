"""Numerics of every sm_100a kernel against the fp32 PyTorch statement of the op."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from ditserve_b200 import ops


def _dev():
    return torch.device("cuda", 0)


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-6)).item()


@pytest.mark.parametrize("M,N,K", [(300, 256, 192), (1000, 1536, 1536), (129, 128, 64), (77, 64, 4096),
                                   (4096, 8960, 1536)])
@pytest.mark.parametrize("epi", ["none", "gelu", "gated", "res"])
def test_gemm_epilogues(M, N, K, epi):
    torch.manual_seed(0)
    d = _dev()
    x = torch.randn(M, K, device=d).bfloat16()
    w = (torch.randn(N, K, device=d) / math.sqrt(K)).bfloat16()
    b = torch.randn(N, device=d).bfloat16()
    kw = {}
    if epi == "gelu":
        kw["act"] = "gelu"
    if epi in ("gated", "res"):
        kw["residual"] = torch.randn(M, N, device=d).bfloat16()
    if epi == "gated":
        rpb = (M + 1) // 2
        kw["gate"] = torch.randn(2, N, device=d)
        kw["rows_per_batch"] = rpb
    y = ops.linear(x, w, b, **kw)
    ref = ops.linear_reference(x.cpu(), w.cpu(), b.cpu(), **{k: (v.cpu() if torch.is_tensor(v) else v)
                                                              for k, v in kw.items()})
    ops.check_status(d)
    assert _rel(y.cpu(), ref) < 1e-2
    torch.testing.assert_close(y.cpu().float(), ref.float(), rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("M,N,K", [(300, 256, 192), (129, 128, 64), (1000, 1536, 1536), (2049, 384, 4104)])
@pytest.mark.parametrize("epi", ["none", "gelu", "gated", "res"])
def test_gemm_cta_pair_epilogues(M, N, K, epi):
    """The CTA-pair (cta_group::2, 256-row tiles) kernel forced on, against the fp32 statement:
    M tails that leave the second CTA of a pair partly or wholly outside the matrix, both pair
    tile widths (N % 256 and N % 128), and a K tail."""
    torch.manual_seed(5)
    d = _dev()
    x = torch.randn(M, K, device=d).bfloat16()
    w = (torch.randn(N, K, device=d) / math.sqrt(K)).bfloat16()
    b = torch.randn(N, device=d).bfloat16()
    kw = {}
    if epi == "gelu":
        kw["act"] = "gelu"
    if epi in ("gated", "res"):
        kw["residual"] = torch.randn(M, N, device=d).bfloat16()
    if epi == "gated":
        kw["gate"] = torch.randn(2, N, device=d)
        kw["rows_per_batch"] = (M + 1) // 2
    y = ops.linear(x, w, b, pair=1, **kw)
    ops.check_status(d)
    ref = ops.linear_reference(x.cpu(), w.cpu(), b.cpu(), **{k: (v.cpu() if torch.is_tensor(v) else v)
                                                              for k, v in kw.items()})
    assert _rel(y.cpu(), ref) < 1e-2
    single = ops.linear(x, w, b, pair=0, **kw)
    assert _rel(y.cpu(), single.cpu()) < 1e-2


@pytest.mark.parametrize("bn", [64, 128, 256])
def test_gemm_tile_widths(bn):
    torch.manual_seed(1)
    d = _dev()
    x = torch.randn(513, 512, device=d).bfloat16()
    w = (torch.randn(512, 512, device=d) / 20).bfloat16()
    y = ops.linear(x, w, None, bn=bn)
    ref = ops.linear_reference(x.cpu(), w.cpu())
    assert _rel(y.cpu(), ref) < 1e-2


def test_gemm_inplace_gated_residual():
    torch.manual_seed(2)
    d = _dev()
    x = torch.randn(640, 1536, device=d).bfloat16()
    w = (torch.randn(1536, 1536, device=d) / 40).bfloat16()
    r = torch.randn(640, 1536, device=d).bfloat16()
    g = torch.randn(1, 1536, device=d)
    ref = ops.linear_reference(x.cpu(), w.cpu(), None, residual=r.cpu(), gate=g.cpu())
    ops.linear(x, w, None, residual=r, gate=g, out=r)
    assert _rel(r.cpu(), ref) < 1e-2


@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("B,Sq,Sk,H", [(2, 300, 300, 2), (1, 128, 512, 3), (1, 1000, 77, 2), (1, 64, 1030, 1)])
def test_attention_dense(D, B, Sq, Sk, H):
    torch.manual_seed(3)
    d = _dev()
    q = torch.randn(B, Sq, H * D, device=d).bfloat16()
    k = torch.randn(B, Sk, H * D, device=d).bfloat16()
    v = torch.randn(B, Sk, H * D, device=d).bfloat16()
    o, lse = ops.attention(q, k, v, H, return_lse=True)
    ro, rlse = ops.attention_reference(q.cpu(), k.cpu(), v.cpu(), H, return_lse=True)
    ops.check_status(d)
    assert _rel(o.cpu(), ro) < 2e-2
    torch.testing.assert_close(o.cpu().float(), ro.float(), rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(lse.cpu().reshape(H, B, Sq).transpose(0, 1), rlse, rtol=1e-3, atol=2e-2)


def test_attention_fused_qkv_view_and_large_logits():
    torch.manual_seed(4)
    d = _dev()
    H, D, S = 4, 128, 777
    qkv = torch.randn(S, 3 * H * D, device=d).bfloat16()
    qkv[:, : H * D] *= 6  # large logits exercise the TMEM O rescale path
    q, k, v = qkv[:, : H * D], qkv[:, H * D: 2 * H * D], qkv[:, 2 * H * D:]
    o = ops.attention(q, k, v, H)
    ro = ops.attention_reference(q.cpu(), k.cpu(), v.cpu(), H)
    assert _rel(o.cpu(), ro) < 2e-2


@pytest.mark.parametrize("D", [64, 128])
def test_attention_varlen(D):
    torch.manual_seed(5)
    d = _dev()
    H = 3
    lens_q = [100, 257, 1024, 5]
    lens_k = [100, 257, 1024, 5]
    cu = torch.tensor([0] + list(torch.tensor(lens_q).cumsum(0)), dtype=torch.int32)
    cuk = torch.tensor([0] + list(torch.tensor(lens_k).cumsum(0)), dtype=torch.int32)
    T, Tk = int(cu[-1]), int(cuk[-1])
    q = torch.randn(T, H * D, device=d).bfloat16()
    k = torch.randn(Tk, H * D, device=d).bfloat16()
    v = torch.randn(Tk, H * D, device=d).bfloat16()
    o = ops.attention(q, k, v, H, cu_seqlens_q=cu.to(d), cu_seqlens_k=cuk.to(d), max_seqlen_q=max(lens_q))
    ro = ops.attention_reference(q.cpu(), k.cpu(), v.cpu(), H, cu_seqlens_q=cu, cu_seqlens_k=cuk)
    assert _rel(o.cpu(), ro) < 2e-2


@pytest.mark.parametrize("D", [1536, 3072])
def test_layernorm_modulate(D):
    torch.manual_seed(6)
    d = _dev()
    x = (torch.randn(2 * 333, D, device=d) * 3 + 1).bfloat16()
    mod = torch.randn(2, 6, D, device=d)
    y = ops.layernorm_modulate(x, scale=mod[:, 1], shift=mod[:, 0], rows_per_batch=333)
    ref = ops.layernorm_modulate_reference(x.cpu(), mod[:, 1].cpu(), mod[:, 0].cpu(), rows_per_batch=333)
    torch.testing.assert_close(y.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)
    w = torch.randn(D, device=d).bfloat16()
    bb = torch.randn(D, device=d).bfloat16()
    y2 = ops.layernorm_modulate(x, weight=w, bias=bb)
    ref2 = ops.layernorm_modulate_reference(x.cpu(), weight=w.cpu(), bias=bb.cpu())
    torch.testing.assert_close(y2.cpu().float(), ref2.float(), rtol=2e-2, atol=2e-2)


def test_rmsnorm_rope_across_heads():
    torch.manual_seed(7)
    d = _dev()
    S, H, D = 300, 12, 128
    qkv = torch.randn(S, 3 * H * D, device=d).bfloat16()
    w = torch.randn(H * D, device=d).bfloat16()
    ang = torch.rand(S, D // 2, device=d) * 6
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    q = qkv[:, : H * D]
    ref = ops.rope_reference(ops.rms_norm_reference(q.cpu(), w.cpu(), 1e-6), cos.cpu(), sin.cpu(), D)
    ops.rmsnorm_rope_(q, w, cos=cos, sin=sin, head_dim=D)
    torch.testing.assert_close(q.cpu().float(), ref.float(), rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("D", [64, 128])
def test_rmsnorm_per_head(D):
    torch.manual_seed(8)
    d = _dev()
    H = 24 if D == 64 else 12
    x = torch.randn(257, H * D, device=d).bfloat16()
    w = torch.randn(D, device=d).bfloat16()
    ref = ops.rms_norm_reference(x.cpu(), w.cpu(), 1e-6, groups=H)
    ops.rmsnorm_rope_(x, w, groups=H, head_dim=D)
    torch.testing.assert_close(x.cpu().float(), ref.float(), rtol=2e-2, atol=3e-2)


def test_sched_step_matches_reference():
    torch.manual_seed(9)
    d = _dev()
    n = 16 * 21 * 8 * 8
    cond = torch.randn(n, device=d).bfloat16()
    unc = torch.randn(n, device=d).bfloat16()
    x = torch.randn(n, device=d)
    last = torch.randn(n, device=d)
    h1 = torch.randn(n, device=d)
    corr = {"last": last, "last_coef": 0.9, "x0_coef": 0.3, "hist": [h1], "hist_coef": [-0.2]}
    pred = {"x": 0.95, "x0": 0.1, "hist": [h1], "hist_coef": [0.05]}
    x0o = torch.empty(n, device=d)
    lo = torch.empty(n, device=d)
    xr = x.cpu().clone()
    x0r = torch.empty(n)
    lr = torch.empty(n)
    ops.sched_step_reference(cond.cpu(), unc.cpu(), 5.0, xr, 0.7,
                             {**corr, "last": last.cpu(), "hist": [h1.cpu()]},
                             {**pred, "hist": [h1.cpu()]}, x0r, lr)
    ops.sched_step(cond, unc, 5.0, x, 0.7, corr, pred, x0o, lo)
    torch.testing.assert_close(x.cpu(), xr, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(x0o.cpu(), x0r, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(lo.cpu(), lr, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("solver", ["unipc", "dpm++", "euler"])
def test_solver_trajectory_through_kernel(solver):
    """A whole solver run with the CUDA step (CFG combine + update) equals the fp32 reference."""
    from ditserve_b200.schedulers import make_scheduler
    torch.manual_seed(11)
    d = _dev()
    n = 16 * 21 * 8 * 8
    x = torch.randn(n, device=d)
    xr = x.cpu().clone()
    a, b = make_scheduler(solver, 6, flow_shift=5.0), make_scheduler(solver, 6, flow_shift=5.0)
    while not a.done:
        cond = torch.randn(n, device=d).bfloat16()
        unc = torch.randn(n, device=d).bfloat16()
        a.step(x, cond, unc, 5.0)
        b.step(xr, cond.cpu(), unc.cpu(), 5.0, kernel=ops.sched_step_reference)
    torch.testing.assert_close(x.cpu(), xr, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("D", [64, 128])
def test_attention_dual_range_segments(D):
    """MMDiT joint attention: each segment = an image block range + a text block range."""
    torch.manual_seed(10)
    d = _dev()
    H = 3
    img = [1024, 256, 4096]
    txt = [333, 333, 77]
    Ti, Tt = sum(img), sum(txt)
    qkv = torch.randn(Ti + Tt, 3 * H * D, device=d).bfloat16()
    q, k, v = qkv[:, :H * D], qkv[:, H * D:2 * H * D], qkv[:, 2 * H * D:]
    segs, io, to = [], 0, Ti
    for a, b in zip(img, txt):
        segs.append((io, io + a, to, to + b, io, io + a, to, to + b))
        io += a
        to += b
    tbl = ops.segment_table(segs)
    o = ops.attention_segments(q, k, v, H, tbl)
    ro = ops.segments_reference(q.cpu(), k.cpu(), v.cpu(), H, tbl)
    ops.check_status(d)
    assert _rel(o.cpu(), ro) < 2e-2


@pytest.mark.parametrize("sources", [2, 3, 4])
def test_attention_multi_source_kv_equals_concatenated(sources):
    """Ring mainloop on one GPU: keys/values split over several sources (as ring peers hold
    them) give the same result as one concatenated key/value set."""
    torch.manual_seed(11)
    d = _dev()
    B, S, H, D = 2, 640, 4, 128
    q = torch.randn(B, S, H * D, device=d).bfloat16()
    ks = [torch.randn(B, S, H * D, device=d).bfloat16() for _ in range(sources)]
    vs = [torch.randn(B, S, H * D, device=d).bfloat16() for _ in range(sources)]
    o = ops.attention(q, ks[0], vs[0], H, kv_extra=list(zip(ks[1:], vs[1:])))
    ref = ops.attention_reference(q.cpu(), torch.cat([k.cpu() for k in ks], 1), torch.cat([v.cpu() for v in vs], 1), H)
    ops.check_status(d)
    assert _rel(o.cpu(), ref) < 2e-2


@pytest.mark.parametrize("chunks", ["1", "4"])
def test_attention_p_chunk_variants(chunks):
    """P handed to the MMA warp in 1 or 4 chunks (DS_ATTN_PCHUNKS; the default is 2) gives the
    same attention; run in a child process since the switch is read once per process."""
    import os
    import subprocess
    import sys
    code = (
        "import torch;from ditserve_b200 import ops\n"
        "torch.manual_seed(3);d=torch.device('cuda',0)\n"
        "for B,Sq,Sk,H,D in ((2,300,300,2,128),(1,129,1030,1,64)):\n"
        "  q=torch.randn(B,Sq,H*D,device=d).bfloat16();k=torch.randn(B,Sk,H*D,device=d).bfloat16()\n"
        "  v=torch.randn(B,Sk,H*D,device=d).bfloat16();o=ops.attention(q,k,v,H);ops.check_status(d)\n"
        "  r=ops.attention_reference(q.cpu(),k.cpu(),v.cpu(),H)\n"
        "  rel=((o.cpu().float()-r.float()).norm()/r.float().norm()).item();assert rel<2e-2,rel\n")
    r = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, DS_ATTN_PCHUNKS=chunks),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.parametrize("B,S,H,D,pattern", [(2, 700, 2, 128, "window"), (1, 1030, 3, 64, "random"),
                                             (1, 2048, 2, 128, "tiles")])
def test_block_sparse_attention_matches_masked_fp32(B, S, H, D, pattern):
    """Only the named 128-key tiles of each 256-row query block are streamed; the result is the
    fp32 softmax attention restricted to the same token pairs (masked tails included)."""
    torch.manual_seed(7)
    dev = torch.device("cuda", 0)
    q = torch.randn(B, S, H * D, device=dev).bfloat16()
    k = torch.randn(B, S, H * D, device=dev).bfloat16()
    v = torch.randn(B, S, H * D, device=dev).bfloat16()
    if pattern == "window":
        bm = ops.sliding_window_block_mask(S, S, 200)
    elif pattern == "tiles":
        bm = ops.tile_window_block_mask((2, 32, 32), (1, 4, 4))
    else:
        g = torch.Generator().manual_seed(3)
        bm = torch.rand(-(-S // 256), -(-S // 128), generator=g) < 0.4
        bm[:, -1] = True  # the ragged last tile is always present
    o, lse = ops.attention(q, k, v, H, block_mask=bm, return_lse=True)
    ops.check_status(dev)
    r, rl = ops.attention_reference(q.cpu(), k.cpu(), v.cpu(), H, return_lse=True, mask=ops.token_mask(bm, S, S))
    rel = ((o.cpu().float() - r.float()).norm() / r.float().norm()).item()
    assert rel < 2e-2, rel
    assert (lse.cpu().view(H, B, S).transpose(0, 1) - rl).abs().max().item() < 2e-2


def test_block_sparse_all_tiles_equals_dense_bitwise():
    torch.manual_seed(8)
    dev = torch.device("cuda", 0)
    B, S, H, D = 2, 900, 2, 128
    q, k, v = (torch.randn(B, S, H * D, device=dev).bfloat16() for _ in range(3))
    full = torch.ones(-(-S // 256), -(-S // 128), dtype=torch.bool)
    assert torch.equal(ops.attention(q, k, v, H, block_mask=full), ops.attention(q, k, v, H))


@pytest.mark.parametrize("B,Sq,Sk,H,D", [(2, 1000, 512, 3, 128), (1, 777, 77, 2, 64)])
def test_short_kv_form_equals_two_tile_form_bitwise(tmp_path, B, Sq, Sk, H, D):
    """Key ranges up to DS_ATTN_SHORT_KV (default 1024) run one Q tile per CTA, two CTAs per SM;
    the per-row arithmetic is the two-tile kernel's, so the outputs agree bit for bit."""
    import os
    import subprocess
    import sys
    torch.manual_seed(9)
    d = _dev()
    q = torch.randn(B, Sq, H * D).bfloat16()
    k = torch.randn(B, Sk, H * D).bfloat16()
    v = torch.randn(B, Sk, H * D).bfloat16()
    torch.save((q, k, v), tmp_path / "in.pt")
    o, lse = ops.attention(q.to(d), k.to(d), v.to(d), H, return_lse=True)
    ops.check_status(d)
    code = ("import torch,sys;from ditserve_b200 import ops\n"
            f"q,k,v=torch.load(sys.argv[1]);d=torch.device('cuda',0)\n"
            f"o,l=ops.attention(q.to(d),k.to(d),v.to(d),{H},return_lse=True);ops.check_status(d)\n"
            "torch.save((o.cpu(),l.cpu()),sys.argv[2])\n")
    r = subprocess.run([sys.executable, "-c", code, str(tmp_path / "in.pt"), str(tmp_path / "out.pt")],
                       env=dict(os.environ, DS_ATTN_SHORT_KV="0"), capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    o2, l2 = torch.load(tmp_path / "out.pt")
    assert torch.equal(o.cpu(), o2) and torch.equal(lse.cpu(), l2)
    ro = ops.attention_reference(q, k, v, H)
    assert _rel(o.cpu(), ro) < 2e-2


@pytest.mark.parametrize("B,S,H", [(1, 4096, 3), (2, 2100, 4), (1, 33000, 1)])
def test_tail_split_matches_unsplit_and_fp32(tmp_path, B, S, H):
    """Units of the last partial round run as key-range parts merged by attention_merge
    (DS_ATTN_SPLIT, on by default); against the unsplit grid (a child process with the split
    off) only the merge's rounding differs, and both match the fp32 statement."""
    import os
    import subprocess
    import sys
    D = 128
    torch.manual_seed(12)
    d = _dev()
    q = torch.randn(B, S, H * D).bfloat16()
    k = torch.randn(B, S, H * D).bfloat16()
    v = torch.randn(B, S, H * D).bfloat16()
    torch.save((q, k, v), tmp_path / "in.pt")
    o, lse = ops.attention(q.to(d), k.to(d), v.to(d), H, return_lse=True)
    ops.check_status(d)
    code = ("import torch,sys;from ditserve_b200 import ops\n"
            "q,k,v=torch.load(sys.argv[1]);d=torch.device('cuda',0)\n"
            f"o,l=ops.attention(q.to(d),k.to(d),v.to(d),{H},return_lse=True);ops.check_status(d)\n"
            "torch.save((o.cpu(),l.cpu()),sys.argv[2])\n")
    r = subprocess.run([sys.executable, "-c", code, str(tmp_path / "in.pt"), str(tmp_path / "out.pt")],
                       env=dict(os.environ, DS_ATTN_SPLIT="0"), capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    o2, l2 = torch.load(tmp_path / "out.pt")
    assert _rel(o.cpu(), o2) < 5e-3, _rel(o.cpu(), o2)
    assert (lse.cpu() - l2).abs().max().item() < 1e-3
    if S <= 4096:
        ro, rl = ops.attention_reference(q, k, v, H, return_lse=True)
        assert _rel(o.cpu(), ro) < 2e-2
        torch.testing.assert_close(lse.cpu().reshape(H, B, S).transpose(0, 1), rl, rtol=1e-3, atol=2e-2)
