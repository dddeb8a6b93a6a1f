"""Wan VAE decode timing: the tcgen05 conv path vs cuDNN, one GPU and row-split over N GPUs.

    python -m ditserve_b200.models.wan.vae_bench                      # 1 GPU
    torchrun --nproc-per-node N -m ditserve_b200.models.wan.vae_bench   # N GPUs, rows split

Decodes a Wan2.1 480p latent (16 x 21 x 60 x 104 -> 3 x 81 x 480 x 832, bf16, random
weights; ``DS_VAE_FRAMES`` latent frames).  One GPU: the module's NCDHW decode (convolutions
by cuDNN through torch, the library baseline) against the channels-last decode on this
package's implicit-GEMM convolution, with their relative L2 difference.  N GPUs: the
channels-last decode with each rank decoding 60 / N latent rows, halo rows exchanged through
NCCL send/recv or stored straight into the neighbours' heap slots; both transports must give
the same video.  Times are CUDA events around the whole decode, after one warm-up decode of
two latent frames, max over ranks.  The reference decodes on rank 0 only (6.91 s for this
tier on A100).
"""
from __future__ import annotations

import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

from .vae import WanVAEDecoder
from .vae_fast import FastDecoder, NCCLHaloCL, PeerHaloCL


def _timed(fn, dev, world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    out = fn()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return out, round(ms, 2)


def main():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    frames = int(os.environ.get("DS_VAE_FRAMES", "21"))
    vae = WanVAEDecoder.random_init(device=dev, dtype=torch.bfloat16, seed=1)
    g = torch.Generator().manual_seed(2)
    z = torch.randn(1, 16, frames, 60, 104, generator=g).to(dev, torch.bfloat16)
    results, outs = {}, {}
    if world == 1:
        for name, fn in (("cudnn_ncdhw", lambda zz: vae.decode(zz)),
                         ("ours_channels_last", lambda zz: FastDecoder(vae).decode(zz))):
            fn(z[:, :, :2])  # warm-up (cuDNN autotune, allocator, weight layouts)
            outs[name], results[name] = _timed(lambda: fn(z), dev, 1)
        a, b = outs["ours_channels_last"].float(), outs["cudnn_ncdhw"].float()
        results["rel_l2_ours_vs_cudnn"] = round(((a - b).norm() / b.norm()).item(), 5)
    else:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        from ...parallel.fused import PeerHalo
        from ...parallel.symm import SymmetricHeap
        heap = SymmetricHeap(80 << 20, dev)
        halos = {"nccl_halo": NCCLHaloCL(), "peer_halo": PeerHaloCL(PeerHalo(heap, tuple(range(world)),
                                                                             max_halo_elems=4 << 20))}
        rows = z.shape[3] // world
        zl = z[:, :, :, rank * rows:(rank + 1) * rows].contiguous()
        for name, halo in halos.items():
            fd = FastDecoder(vae, halo)
            fd.decode(zl[:, :, :2])
            outs[name], results[name] = _timed(lambda: fd.decode(zl), dev, world)
        same = torch.equal(outs["nccl_halo"], outs["peer_halo"])
        flag = torch.tensor([1 if same else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        results["transports_bitwise_equal"] = bool(flag.item())
    if rank == 0:
        print(json.dumps({"vae_decode_ms": results, "world": world, "frames": frames,
                          "output_shape": [1, 3, 1 + 4 * (frames - 1), 480, 832]}))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
