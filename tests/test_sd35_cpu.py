"""SD3.5 MMDiT (tiny config, fp32, CPU): packing equivalence, continuous batching, resume."""
import torch

from ditserve_b200.models.sd35.model import SD35_TINY, SD35Transformer
from ditserve_b200.models.sd35.runtime import SD35Engine


def _engine():
    return SD35Engine(SD35_TINY, device="cpu", dtype=torch.float32, seed=2)


def test_packed_batch_equals_individual_forwards():
    m = SD35Transformer.random_init(SD35_TINY, dtype=torch.float32, seed=1)
    cfg = SD35_TINY
    torch.manual_seed(0)
    lat = [torch.randn(16, 16, 16), torch.randn(16, 8, 12), torch.randn(16, 4, 4)]
    ctx = [torch.randn(7, cfg.joint_dim), torch.randn(5, cfg.joint_dim), torch.randn(9, cfg.joint_dim)]
    pool = [torch.randn(cfg.pooled_dim) for _ in range(3)]
    t = [900.0, 500.0, 10.0]
    packed = m.forward_packed(lat, t, ctx, pool)
    for i in range(3):
        solo = m.forward_packed([lat[i]], [t[i]], [ctx[i]], [pool[i]])[0]
        torch.testing.assert_close(packed[i], solo, rtol=1e-5, atol=1e-5)


def test_continuous_batching_late_join_matches_solo_runs():
    e = _engine()
    specs = [dict(height=128, width=128, steps=4, seed=1), dict(height=64, width=96, steps=3, seed=2),
             dict(height=64, width=64, steps=2, seed=3, guidance=1.0)]
    solo = [e.run(e.prepare(s)) for s in specs]
    a, b, c = (e.prepare(s) for s in specs)
    e.advance_batch([a])            # a alone
    e.advance_batch([a, b])         # b joins late
    e.advance_batch([a, b, c])      # c joins; heterogeneous resolutions and CFG on/off
    e.advance_batch([a, b, c])      # b and c finish (early exit)
    while not a.done:
        e.advance_batch([a, b, c])
    for got, want in zip((a, b, c), solo):
        torch.testing.assert_close(got.latents, want.latents, rtol=1e-4, atol=1e-4)


def test_snapshot_restore_is_bitwise():
    e = _engine()
    s = e.prepare(dict(height=64, width=64, steps=3, seed=9))
    full = e.run(e.prepare(dict(height=64, width=64, steps=3, seed=9)))
    e.advance_batch([s])
    r = e.restore(e.snapshot(s))
    e.run(r)
    assert torch.equal(r.latents, full.latents)


def test_sd35_block_export_import(tmp_path):
    from ditserve_b200.models.sd35.backend import SD35Backend
    a = SD35Backend({"model": "sd3.5-tiny", "device": "cpu", "transfer_dir": str(tmp_path)})
    b = SD35Backend({"model": "sd3.5-tiny", "device": "cpu", "transfer_dir": str(tmp_path)})
    a.prepare(dict(id=1, state_id="i", spec=dict(height=64, width=64, steps=3, seed=2)))
    a.advance(dict(id=2, state_id="i", steps=1))
    pk = a.block_export(dict(id=3, state_id="i"))
    b.block_import(dict(id=4, state_id="i", path=pk["path"], manifest=pk["manifest"]))
    a.advance(dict(id=5, state_id="i", steps=2))
    b.advance(dict(id=6, state_id="i", steps=2))
    import torch
    assert torch.equal(a.states["i"].latents, b.states["i"].latents)


def test_sd35_vae_decoder_layout_and_finish(tmp_path):
    import torch
    from ditserve_b200.models.sd35.backend import SD35Backend
    from ditserve_b200.models.sd35.vae import SD35VAEDecoder
    full = SD35VAEDecoder()
    keys = set(full.state_dict())
    for k in ("decoder.conv_in.weight", "decoder.mid_block.attentions.0.to_q.weight",
              "decoder.mid_block.attentions.0.to_out.0.bias", "decoder.mid_block.resnets.1.conv2.weight",
              "decoder.up_blocks.0.upsamplers.0.conv.weight", "decoder.up_blocks.2.resnets.0.conv_shortcut.weight",
              "decoder.up_blocks.3.resnets.2.norm2.weight", "decoder.conv_norm_out.weight", "decoder.conv_out.bias"):
        assert k in keys, k
    assert "decoder.up_blocks.3.upsamplers.0.conv.weight" not in keys
    vae = SD35VAEDecoder.random_init(dtype=torch.float32, channels=(32, 32, 64, 64))
    img = vae.decode(torch.randn(1, 16, 8, 8))
    assert img.shape == (1, 3, 64, 64) and img.abs().max() <= 1
    b = SD35Backend({"model": "sd3.5-tiny", "device": "cpu", "transfer_dir": str(tmp_path),
                     "vae_channels": [32, 32, 64, 64], "decode_images": True})
    b.prepare(dict(id=1, state_id="i", spec=dict(height=64, width=64, steps=1, seed=2)))
    b.advance(dict(id=2, state_id="i", steps=1))
    out = b.finish(dict(id=3, state_id="i", output_mode="digest"))
    assert out["shape"] == [1, 3, 64, 64]
