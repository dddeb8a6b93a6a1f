"""Channels-last VAE decode (the path of the implicit-GEMM tcgen05 convolution) against the
module's own NCDHW decode: exact on CPU in fp32 (same weights), both Wan2.1 and Wan2.2
decoders; row-split patch parallelism over a Gloo world of 2 equal to the single-rank decode;
and on a B200 the bf16 conv-kernel decode against the fp32 CPU statement."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ditserve_b200.models.wan.vae import WanVAEDecoder
from ditserve_b200.models.wan.vae_fast import FastDecoder, NCCLHaloCL

VARIANTS = {"wan2.1": dict(z_dim=16, base=32, residual=False, patch=1),
            "wan2.2": dict(z_dim=48, base=64, residual=True, patch=2)}


def _vae(variant, seed=2):
    torch.manual_seed(seed)
    m = WanVAEDecoder(**VARIANTS[variant]).eval()
    with torch.no_grad():  # weights on the bf16 grid, so a bf16 copy holds the same values
        for p in m.parameters():
            p.copy_(p.bfloat16().float())
    return m


def _z(variant, h=6, w=8):
    g = torch.Generator().manual_seed(7)
    return torch.randn(1, VARIANTS[variant]["z_dim"], 3, h, w, generator=g)


@pytest.mark.parametrize("variant", ["wan2.1", "wan2.2"])
def test_channels_last_decode_equals_module_decode(variant):
    m = _vae(variant)
    z = _z(variant)
    ref = m.decode(z)
    out = FastDecoder(m).decode(z)
    assert out.shape == ref.shape
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = _vae("wan2.1")
        z = _z("wan2.1")
        rows = z.shape[3] // world
        part = FastDecoder(m, NCCLHaloCL()).decode(z[:, :, :, rank * rows:(rank + 1) * rows].contiguous())
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        if rank == 0:
            out["pp"] = torch.cat(parts, dim=3)
    finally:
        dist.destroy_process_group()


def test_row_split_decode_equals_single_rank():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
    ref = FastDecoder(_vae("wan2.1")).decode(_z("wan2.1"))
    torch.testing.assert_close(out["pp"], ref, rtol=1e-4, atol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("variant", ["wan2.1", "wan2.2"])
def test_conv_kernel_decode_matches_fp32_cpu(variant):
    m = _vae(variant)
    z = _z(variant, h=8, w=12)
    ref = m.decode(z)
    g = WanVAEDecoder(**VARIANTS[variant]).to("cuda", torch.bfloat16).eval()
    g.load_state_dict({k: v.to(torch.bfloat16) for k, v in m.state_dict().items()})
    from ditserve_b200 import ops
    ops.launch_counts(reset=True)
    out = FastDecoder(g).decode(z.cuda())
    ops.check_status(torch.device("cuda", 0))
    assert ops.launch_counts().get("conv", 0) > 0, "the decode must run on the conv kernel"
    assert out.shape == ref.shape
    rel = ((out.float().cpu() - ref).norm() / ref.norm()).item()
    assert rel < 5e-2, rel


def test_decode_halo_transport_choice():
    from ditserve_b200.models.wan.backend import decode_halo_transport
    assert decode_halo_transport("auto", 2, "cuda") == "peer"
    assert decode_halo_transport("auto", 4, "cuda") == "nccl"
    assert decode_halo_transport("peer", 8, "cuda") == "peer"
    assert decode_halo_transport("auto", 2, "cpu") == "nccl"
    import pytest
    with pytest.raises(ValueError):
        decode_halo_transport("nvls", 2, "cuda")
