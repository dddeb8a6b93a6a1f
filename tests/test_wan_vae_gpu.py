"""Wan VAE decoder on the GPU (bf16) against its fp32 CPU statement, and chunked resume."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from ditserve_b200.models.wan.vae import ChunkedDecode, WanVAEDecoder


def test_vae_decode_gpu_matches_cpu():
    cpu = WanVAEDecoder.random_init(dtype=torch.float32, seed=3)
    gpu = WanVAEDecoder.random_init(device="cuda", dtype=torch.bfloat16, seed=3)
    gpu.load_state_dict({k: v.to(torch.bfloat16) for k, v in cpu.state_dict().items()})
    z = torch.randn(1, 16, 3, 8, 12, generator=torch.Generator().manual_seed(1))
    ref = cpu.decode(z)
    out = gpu.decode(z.cuda())
    assert out.shape == ref.shape == (1, 3, 9, 64, 96)
    rel = ((out.float().cpu() - ref).norm() / ref.norm()).item()
    assert rel < 0.1, rel
    d = ChunkedDecode(gpu, z.cuda())
    d.step()
    d.step(5)
    assert torch.equal(d.result(), out)
