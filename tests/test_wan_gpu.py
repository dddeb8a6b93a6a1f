"""Correctness gates of the Wan product path on the sm_100a kernels (one GPU).

* a tiny Wan DiT forward on CUDA (bf16, tcgen05 GEMMs and attention) against the fp32 CPU
  statement of the same weights;
* the same-parallelism gate through the CUDA kernels: an uninterrupted 4-step UniPC run, a
  run paused at a step boundary (snapshot, serialise, restore) and a run cut into block
  quanta (doorbell stop, continuation packet export/import) end on bitwise equal latents
  (the reference's block-preemption exactness check: benchmarks/native_exact.py);
* the fused Ulysses kernels as one-member groups (qkv_scatter: RMS q/k norm + RoPE + staging
  copy; attention_scatter: attention whose epilogue stores rows by owner) against the fp32
  statements of norm, RoPE and attention;
* guard bands: outputs written through views of larger buffers leave the surrounding
  sentinel region untouched on M/N/K tail shapes.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from ditserve_b200 import ops
from ditserve_b200.models.wan import config as wcfg
from ditserve_b200.models.wan.config import WanConfig
from ditserve_b200.models.wan.model import WanTransformer
from ditserve_b200.models.wan.runtime import WanEngine

CFG = WanConfig("wan-gpu-gate", dim=512, heads=4, ffn_dim=1024, layers=2, in_channels=16, out_channels=16,
                text_dim=256, text_len=64)
wcfg.CONFIGS[CFG.name] = CFG
# 240x240, 9 frames -> latent 16 x 3 x 30 x 30 -> 675 tokens (not a multiple of the 128-row tiles)
SPEC = dict(model=CFG.name, height=240, width=240, frames=9, steps=4, guidance=5.0, seed=11)


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def test_wan_forward_matches_fp32_cpu_statement():
    dev = torch.device("cuda", 0)
    m = WanTransformer.random_init(CFG, device=dev, dtype=torch.bfloat16, seed=3)
    g = torch.Generator().manual_seed(5)
    lat = torch.randn(2, 16, 3, 30, 30, generator=g)
    ctx = torch.randn(2, CFG.text_len, CFG.text_dim, generator=g)
    t = torch.tensor([900.0, 900.0])
    with torch.inference_mode():
        out = m(lat.to(dev, torch.bfloat16), t.to(dev), ctx.to(dev, torch.bfloat16))
    ops.check_status(dev)
    mc = WanTransformer(CFG)
    mc.load_state_dict({k: v.float().cpu() for k, v in m.state_dict().items()})
    mc.prepare()
    with torch.inference_mode():
        ref = mc(lat, t, ctx)
    assert out.shape == ref.shape
    assert torch.isfinite(out.float()).all()
    assert _rel(out, ref) < 5e-2, _rel(out, ref)


def test_same_parallelism_gate_is_bitwise_on_the_cuda_kernels():
    dev = torch.device("cuda", 0)
    e = WanEngine(CFG, device=dev, seed=1)
    full = e.run(e.prepare(SPEC)).latents.clone()
    # step-boundary pause: snapshot after 2 steps, serialise, restore, finish
    st = e.prepare(SPEC)
    e.step(st)
    e.step(st)
    resumed = e.restore(e.unpack(e.pack(e.snapshot(st))))
    e.run(resumed)
    assert torch.equal(resumed.latents, full), "pause/resume changed the latents"
    # block quanta: a doorbell stop after one block, a continuation packet across the cut,
    # then quanta of one block and of the rest of the step
    st = e.prepare(SPEC)
    rang = {"n": 0}

    def bell():
        rang["n"] += 1
        return rang["n"] == 1

    r = e.advance(st, bell=bell, check_every=1)
    assert r["doorbell_stop"] and r["blocks"] == 1 and not r["step_completed"]
    blob, digest = e.export_packet(st)
    st2 = e.import_packet(blob, digest)
    e.advance(st2, blocks=1)
    while not st2.done:
        e.advance(st2, blocks=1)
        if not st2.done:
            e.advance(st2)
    ops.check_status(dev)
    assert torch.equal(st2.latents.cpu(), full.cpu()), "block quanta changed the latents"


def _fp32_norm_rope(x, w, eps, cos, sin, heads, hd, seq):
    x = x.float()
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    pos = torch.arange(y.shape[0], device=y.device) % seq
    c, s = cos[pos].repeat(1, heads), sin[pos].repeat(1, heads)
    out = torch.empty_like(y)
    out[:, 0::2] = y[:, 0::2] * c - y[:, 1::2] * s
    out[:, 1::2] = y[:, 0::2] * s + y[:, 1::2] * c
    return out


def _fp32_attention(q, k, v, batch, seq, heads, hd):
    qh = q.float().view(batch, seq, heads, hd).transpose(1, 2)
    kh = k.float().view(batch, seq, heads, hd).transpose(1, 2)
    vh = v.float().view(batch, seq, heads, hd).transpose(1, 2)
    p = torch.softmax(qh @ kh.transpose(-1, -2) / math.sqrt(hd), dim=-1)
    return (p @ vh).transpose(1, 2).reshape(batch * seq, heads * hd)


@pytest.mark.parametrize("heads,hd,seq", [(12, 128, 333), (8, 64, 400), (4, 128, 2100)])
def test_fused_ulysses_kernels_as_a_one_member_group(heads, hd, seq):
    # (4, 128, 2100): 72 query-block units on 148 SMs, so the attention grid runs key-range
    # parts and the merge kernel stores the rows through the peer-store path
    dev = torch.device("cuda", 0)
    ext = ops.ext()
    batch, eps = 2, 1e-6
    width = heads * hd
    g = torch.Generator().manual_seed(heads)
    qkv = torch.randn(batch * seq, 3 * width, generator=g).bfloat16().to(dev)
    wq = (1 + 0.1 * torch.randn(width, generator=g)).bfloat16().to(dev)
    wk = (1 + 0.1 * torch.randn(width, generator=g)).bfloat16().to(dev)
    ang = torch.rand(seq, hd // 2, generator=g) * 4
    cos, sin = ang.cos().contiguous().to(dev), ang.sin().contiguous().to(dev)
    stage_bytes = batch * seq * 3 * width * 2
    out_bytes = batch * seq * width * 2
    flag = max(4096, int(ext.FLAG_BYTES))
    heap, _ = ext.symm_alloc(flag + stage_bytes + out_bytes + 4096, 0)
    base = heap.data_ptr()
    recv_off, o_off = flag, flag + stage_bytes
    st = ops.status_word(dev)
    ext.qkv_scatter(qkv, wq, wk, eps, cos, sin, seq, heads, hd, 0, [base], int(1e9), recv_off, 0)
    staged = heap[recv_off:recv_off + stage_bytes].view(torch.bfloat16).view(batch * seq, 3 * width)
    q, k, v = staged[:, :width], staged[:, width:2 * width], staged[:, 2 * width:]
    ext.attention_scatter(q, k, v, batch, seq, heads, hd, 1.0 / math.sqrt(hd), 0, [base], int(1e9), o_off, seq, 0,
                          width, st, [], [])
    torch.cuda.synchronize()
    ops.check_status(dev)
    x = qkv.float()
    rq = _fp32_norm_rope(x[:, :width], wq, eps, cos, sin, heads, hd, seq)
    rk = _fp32_norm_rope(x[:, width:2 * width], wk, eps, cos, sin, heads, hd, seq)
    assert _rel(q, rq) < 1e-2 and _rel(k, rk) < 1e-2
    assert torch.equal(v, qkv[:, 2 * width:]), "v must be staged unchanged"
    o = heap[o_off:o_off + out_bytes].view(torch.bfloat16).view(batch * seq, width)
    ro = _fp32_attention(rq, rk, x[:, 2 * width:], batch, seq, heads, hd)
    assert _rel(o, ro) < 2e-2, _rel(o, ro)


SENTINEL = 1024.0  # exactly representable in bf16, far outside what the ops write here


@pytest.mark.parametrize("pair", [0, 1])
@pytest.mark.parametrize("M,N,K,epi", [(300, 192, 200, "none"), (129, 256, 72, "gelu"), (1000, 384, 1536, "res"),
                                       (77, 512, 4104, "gated")])
def test_gemm_leaves_the_guard_band_untouched(M, N, K, epi, pair):
    dev = torch.device("cuda", 0)
    torch.manual_seed(M)
    x = torch.randn(M, K, device=dev).bfloat16()
    w = (torch.randn(N, K, device=dev) / math.sqrt(K)).bfloat16()
    b = torch.randn(N, device=dev).bfloat16()
    buf = torch.full((M + 16, N + 64), SENTINEL, device=dev, dtype=torch.bfloat16)
    out = buf[8:8 + M, 32:32 + N]
    kw = {}
    if epi == "gelu":
        kw["act"] = "gelu"
    if epi in ("res", "gated"):
        kw["residual"] = torch.randn(M, N, device=dev).bfloat16()
    if epi == "gated":
        kw["gate"] = torch.randn(1, N, device=dev)
    ops.linear(x, w, b, out=out, pair=pair, **kw)
    torch.cuda.synchronize()
    ops.check_status(dev)
    band = buf.clone()
    band[8:8 + M, 32:32 + N] = SENTINEL
    assert torch.all(band == SENTINEL), "the GEMM wrote outside its output view"
    ref = ops.linear_reference(x.cpu(), w.cpu(), b.cpu(), **{k: (v.cpu() if torch.is_tensor(v) else v)
                                                              for k, v in kw.items()})
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("B,Sq,Sk,H,D", [(2, 300, 300, 2, 128), (1, 129, 77, 3, 64), (1, 1000, 512, 1, 128)])
def test_attention_leaves_the_guard_band_untouched(B, Sq, Sk, H, D):
    dev = torch.device("cuda", 0)
    torch.manual_seed(Sq)
    W = H * D
    q = torch.randn(B * Sq, W, device=dev).bfloat16()
    k = torch.randn(B * Sk, W, device=dev).bfloat16()
    v = torch.randn(B * Sk, W, device=dev).bfloat16()
    buf = torch.full((B * Sq + 16, W + 64), SENTINEL, device=dev, dtype=torch.bfloat16)
    out = buf[8:8 + B * Sq, 32:32 + W]
    ops.attention(q.view(B, Sq, W), k.view(B, Sk, W), v.view(B, Sk, W), H, out=out)
    torch.cuda.synchronize()
    ops.check_status(dev)
    band = buf.clone()
    band[8:8 + B * Sq, 32:32 + W] = SENTINEL
    assert torch.all(band == SENTINEL), "attention wrote outside its output view"
    ref = ops.attention_reference(q.view(B, Sq, W).cpu(), k.view(B, Sk, W).cpu(), v.view(B, Sk, W).cpu(), H)
    assert _rel(out.reshape(B, Sq, W), ref) < 2e-2


def test_inplace_norm_rope_leaves_neighbouring_columns_untouched():
    """q is normalised in place inside the fused QKV buffer; the k and v columns beside it
    must come out bit for bit as they went in."""
    dev = torch.device("cuda", 0)
    torch.manual_seed(9)
    rows, heads, hd = 777, 12, 128
    width = heads * hd
    qkv = torch.randn(rows, 3 * width, device=dev).bfloat16()
    before = qkv.clone()
    w = (1 + 0.1 * torch.randn(width, device=dev)).bfloat16()
    ang = torch.rand(rows, hd // 2, device=dev)
    ops.rmsnorm_rope_(qkv[:, :width], w, eps=1e-6, cos=ang.cos().contiguous(), sin=ang.sin().contiguous(),
                      rows_per_batch=rows, head_dim=hd)
    torch.cuda.synchronize()
    ops.check_status(dev)
    assert torch.equal(qkv[:, width:], before[:, width:])
    ref = _fp32_norm_rope(before[:, :width], w, 1e-6, ang.cos(), ang.sin(), heads, hd, rows)
    assert _rel(qkv[:, :width], ref) < 1e-2


def test_single_launch_qk_norm_equals_two_launches():
    """q and k normalised + rotated in one launch give the same bits as one launch each, and
    leave v untouched."""
    dev = torch.device("cuda", 0)
    torch.manual_seed(11)
    rows, heads, hd = 1000, 12, 128
    width = heads * hd
    qkv = torch.randn(rows, 3 * width, device=dev).bfloat16()
    wq = (1 + 0.1 * torch.randn(width, device=dev)).bfloat16()
    wk = (1 + 0.1 * torch.randn(width, device=dev)).bfloat16()
    ang = torch.rand(500, hd // 2, device=dev)
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    a, b = qkv.clone(), qkv.clone()
    ops.rmsnorm_rope_qk_(a, wq, wk, eps=1e-6, cos=cos, sin=sin, rows_per_batch=500, head_dim=hd)
    ops.rmsnorm_rope_(b[:, :width], wq, eps=1e-6, cos=cos, sin=sin, rows_per_batch=500, head_dim=hd)
    ops.rmsnorm_rope_(b[:, width:2 * width], wk, eps=1e-6, cos=cos, sin=sin, rows_per_batch=500, head_dim=hd)
    torch.cuda.synchronize()
    ops.check_status(dev)
    assert torch.equal(a, b)
    assert torch.equal(a[:, 2 * width:], qkv[:, 2 * width:])


def test_live_exactness_harness_on_the_cuda_kernels():
    """The exactness tool's live mode: seeded cuts at random block boundaries (continuation
    packets, step-boundary snapshots) end on the uninterrupted latents bit for bit."""
    from ditserve_b200.evaluation import exactness
    out = exactness.live_check(device="cuda", schedules=2, cuts=3, seed=2, spec=dict(SPEC, steps=3))
    assert out["status"] == "completed", out["runs"]
