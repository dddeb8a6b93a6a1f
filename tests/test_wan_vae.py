"""Wan causal VAE decoder (CPU, fp32): shapes, resumable chunked decode, patch-parallel
decode over Gloo world 2 equal to the single-rank decode."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ditserve_b200.models.wan.vae import ChunkedDecode, PatchParallel, WanVAEDecoder, split_latent


def _vae():
    return WanVAEDecoder.random_init(dtype=torch.float32, seed=3)


def _z():
    g = torch.Generator().manual_seed(5)
    return torch.randn(1, 16, 3, 4, 6, generator=g)


def test_decode_shapes_and_chunked_resume():
    vae = _vae()
    z = _z()
    full = vae.decode(z)
    assert full.shape == (1, 3, 9, 32, 48)
    assert full.abs().max() <= 1.0
    d = ChunkedDecode(vae, z)
    d.step()  # pause after the first latent frame
    d2 = d.step(2)
    assert d2.done
    assert torch.equal(d.result(), full)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        vae = _vae()
        halo = PatchParallel(axis=4)
        part = vae.decode(split_latent(_z(), halo), halo)
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        if rank == 0:
            out["pp"] = torch.cat(parts, dim=4)
    finally:
        dist.destroy_process_group()


def test_patch_parallel_decode_equals_single_rank():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
    ref = _vae().decode(_z())
    torch.testing.assert_close(out["pp"], ref, rtol=1e-4, atol=1e-4)


def test_wan22_vae_residual_decoder_chunked_equals_whole():
    import torch
    from ditserve_b200.models.wan.vae import ChunkedDecode, DupUp3D, WanVAEDecoder
    m = WanVAEDecoder.random_init(dtype=torch.float32, variant="wan2.2")
    keys = set(m.state_dict())
    for k in ("decoder.up_blocks.0.upsampler.time_conv.weight", "decoder.up_blocks.2.upsampler.resample.1.weight",
              "decoder.conv_out.weight", "post_quant_conv.weight", "decoder.mid_block.attentions.0.to_qkv.weight"):
        assert k in keys, k
    assert "decoder.up_blocks.3.upsampler.resample.1.weight" not in keys
    assert m.decoder.conv_out.out_channels == 12
    g = torch.Generator().manual_seed(0)
    z = torch.randn(1, 48, 3, 2, 3, generator=g)
    whole = m.decode(z)
    assert whole.shape == (1, 3, 9, 32, 48)
    dec = ChunkedDecode(m, z)
    dec.step(1)
    dec.step(2)
    assert torch.equal(dec.result(), whole)
    # the shortcut's first chunk keeps one frame per latent frame, later chunks double time
    d = DupUp3D(8, 4, 2, 2)
    x = torch.randn(1, 8, 1, 2, 2)
    assert d(x).shape == (1, 4, 2, 4, 4) and d(x, first_chunk=True).shape == (1, 4, 1, 4, 4)
