"""Approximate-mode extras on the tiny Wan (CPU): CFG folding, block-residual reuse, INT8 codec."""
import torch

from ditserve_b200.models.approx import (BlockResidualCache, CFGFolding, dequantize_int8, packet_bytes,
                                         quantize_int8)
from ditserve_b200.models.wan.runtime import WanEngine

SPEC = dict(model="wan-tiny", height=64, width=64, frames=13, steps=12, guidance=5.0, seed=2)


def _cos(a, b):
    a, b = a.flatten().double(), b.flatten().double()
    return (a @ b / (a.norm() * b.norm())).item()


def test_cfg_folding_skips_uncond_and_stays_close():
    e = WanEngine("wan-tiny", device="cpu", dtype=torch.float32, seed=1)
    exact = e.run(e.prepare(SPEC))
    st = e.prepare(SPEC)
    fold = CFGFolding(SPEC["steps"], warm_frac=0.4, threshold=0.5, fold_span=2)
    with torch.inference_mode():
        while not st.done:
            br, lat, t, ctx = e._inputs(st)
            if fold.fold_now(st.step):
                pred = e.model(lat[:1], t[:1], ctx[:1])
                v = fold.combine(st.step, st.spec.guidance, pred[0], None)
            else:
                pred = e.model(lat, t, ctx)
                v = fold.combine(st.step, st.spec.guidance, pred[0], pred[1])
            st.scheduler.step(st.latents.view(-1), v.reshape(-1), None, 1.0)
            st.step += 1
    assert fold.folded_steps > 0 and fold.full_steps + fold.folded_steps == SPEC["steps"]
    assert _cos(st.latents, exact.latents) > 0.9


def test_block_residual_cache_reuses_middle_blocks():
    from ditserve_b200.models.wan.config import WanConfig
    from ditserve_b200.models.wan import config as wcfg
    cfg = WanConfig("wan-tiny6", dim=128, heads=4, ffn_dim=512, layers=6, in_channels=16, out_channels=16,
                    text_dim=64, text_len=16)
    wcfg.CONFIGS[cfg.name] = cfg
    e = WanEngine(cfg, device="cpu", dtype=torch.float32, seed=1)
    spec = dict(SPEC, model=cfg.name)
    exact = e.run(e.prepare(spec))
    st = e.prepare(spec)
    cache = BlockResidualCache(cfg.layers, front=1, back=1, threshold=0.5)
    with torch.inference_mode():
        while not st.done:
            br, lat, t, ctx = e._inputs(st)
            pk = e.model.begin(lat, t, ctx)
            cache.run_wan(e.model, pk)
            pred = e.model.predict(pk)
            e.apply(st, pred[0], pred[1])
    assert cache.skipped_blocks > 0
    assert _cos(st.latents, exact.latents) > 0.85


def test_int8_ring_codec():
    x = torch.randn(64, 12 * 128).bfloat16()
    q, s = quantize_int8(x, 128)
    y = dequantize_int8(q, s, 128)
    assert _cos(x.float(), y.float()) > 0.999
    assert packet_bytes(1, 1, 128, True) == 132 and packet_bytes(1, 1, 128, False) == 256


def test_sd35_block_cache_reuse():
    import torch
    from ditserve_b200.models.approx import BlockResidualCache
    from ditserve_b200.models.sd35.model import SD35_TINY, SD35Transformer
    m = SD35Transformer.random_init(SD35_TINY, device="cpu", dtype=torch.float32, seed=0)
    m.prepare()
    g = torch.Generator().manual_seed(0)
    lat = [torch.randn(SD35_TINY.in_channels, 32, 32, generator=g)]
    ctx = [torch.randn(8, SD35_TINY.joint_dim, generator=g)]
    pooled = [torch.randn(SD35_TINY.pooled_dim, generator=g)]
    layers = SD35_TINY.layers
    if layers < 3:
        import pytest
        pytest.skip("tiny config has too few blocks for a middle range")
    cache = BlockResidualCache(layers, front=1, back=1, threshold=1.0, max_reuse=2)
    exact = m.forward_packed(lat, [500.0], ctx, pooled)[0]
    first = m.forward_packed(lat, [500.0], ctx, pooled, cache=cache)[0]
    assert torch.allclose(first, exact, atol=1e-5)  # nothing cached yet: exact
    again = m.forward_packed(lat, [499.0], ctx, pooled, cache=cache)[0]
    assert cache.skipped_blocks == layers - 2
    assert torch.isfinite(again).all()


def test_wan_engine_cfg_folding_skips_uncond_branch():
    import torch
    from ditserve_b200.models.wan.runtime import WanEngine
    e = WanEngine("wan-tiny", device="cpu", dtype=torch.float32)
    base = dict(model="wan-tiny", height=64, width=64, frames=5, steps=6, seed=3, guidance=5.0)
    exact = e.run(e.prepare(base))
    st = e.prepare(dict(base, cfg_fold={"warm_frac": 0.0, "threshold": 10.0, "fold_span": 1}))
    calls = []
    orig = e.model.begin

    def spy(lat, t, ctx, pctx=None):
        calls.append(lat.shape[0])
        return orig(lat, t, ctx, pctx)
    e.model.begin = spy
    e.run(st)
    assert st.fold.folded_steps >= 2 and 1 in calls       # some steps ran the conditional branch only
    rel = ((st.latents - exact.latents).norm() / exact.latents.norm()).item()
    assert torch.isfinite(st.latents).all() and rel < 1.0
