"""Wan VAE decode: single GPU vs patch-parallel (NCCL halo baseline vs peer-memory halo).

    python -m ditserve_b200.models.wan.vae_bench                      # 1 GPU
    torchrun --nproc-per-node N -m ditserve_b200.models.wan.vae_bench   # N GPUs, split along W

Decodes a Wan2.1 480p latent (16 x 21 x 60 x 104 -> 3 x 81 x 480 x 832, bf16, random
weights).  Multi-GPU runs check that both transports give the same video as each other
and report device time (max over ranks).  The reference decodes on rank 0 only
(6.91 s for this tier on A100).
"""
from __future__ import annotations

import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

from .vae import PatchParallel, WanVAEDecoder, split_latent


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
    results = {}
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        base = PatchParallel(axis=4)
        from ...parallel.fused import PeerHalo
        from ...parallel.symm import SymmetricHeap
        heap = SymmetricHeap(64 << 20, dev)
        peer = PeerHalo(heap, tuple(range(world)), axis=4, baseline=base)
        halos = {"nccl": base, "peer": peer}
    else:
        halos = {"single": None}
    outs = {}
    for name, halo in halos.items():
        zl = split_latent(z, halo) if halo is not None else z
        vae.decode(zl[:, :, :2], halo)  # warm-up (cuDNN autotune, allocator)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        out = vae.decode(zl, halo)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        results[name] = round(ms, 2)
        outs[name] = out
    if world > 1:
        same = torch.equal(outs["nccl"], outs["peer"])
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
