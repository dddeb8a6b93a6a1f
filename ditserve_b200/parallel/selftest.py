"""Multi-GPU self-check: fused peer-memory collectives vs the NCCL path.

    torchrun --nproc-per-node N -m ditserve_b200.parallel.selftest [--steps 2] [--tiny]

Runs the same seeded Wan request with the NCCL plans and with the fused plans of
the default form for N GPUs (N=2 cfg2, N=4 cfg2sp2, N=8 cfg2sp4) and checks that
the latents are bitwise equal (the fused kernels move the same bytes and apply
the same arithmetic), then reports per-step device times of both paths
(max over ranks).  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--tiny", action="store_true", help="small 2-block model at 240p (fast)")
    ap.add_argument("--form", default=None, help="parallel form (default: cfg2 x Ulysses over the world)")
    ap.add_argument("--record", default=None, help="append the timing to this collective-path table (autotune)")
    args = ap.parse_args()
    from ..models.wan.config import WAN21_T2V_1_3B, WanConfig
    from ..models.wan import config as wcfg
    from ..models.wan.runtime import WanEngine, WanSpec
    from ..ops import check_status
    from .layout import FixedLayout, default_form
    from .runtime import build_parallel

    rank, world, local = (int(os.environ[k]) for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    cfg = WAN21_T2V_1_3B
    if args.tiny:
        cfg = WanConfig("wan-selftest", dim=1536, heads=12, ffn_dim=2048, layers=2, in_channels=16, out_channels=16)
        wcfg.CONFIGS[cfg.name] = cfg
    # tiny: 21 x 16 x 28 = 9408 tokens, divisible by every SP degree up to 8
    spec = WanSpec(model=cfg.name, height=256 if args.tiny else 480, width=448 if args.tiny else 832, frames=81,
                   steps=10, guidance=5.0, seed=3)
    lat = spec.latent_shape()
    from .layout import Form
    form = Form.parse(args.form) if args.form else default_form(world)
    layout = FixedLayout(tuple(range(world)), form)
    out = {}
    for path in ("nccl", "fused"):
        pctx, plan = build_parallel(layout, rank, dev, attention=path, seq_local=cfg.tokens(lat) // form.sp,
                                    cfg=cfg, pred_numel=lat[0] * lat[1] * lat[2] * lat[3])
        eng = WanEngine(cfg, device=dev, pctx=pctx, cfg_plan=plan, seed=5)
        st = eng.prepare(spec)
        eng.step(st)  # warm-up step (also the first compared step)
        torch.cuda.synchronize()
        dist.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps - 1):
            eng.step(st)
        t1.record()
        torch.cuda.synchronize()
        check_status(dev)
        ms = t0.elapsed_time(t1) / max(1, args.steps - 1)
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[path] = dict(latent=st.latents.detach().clone(), ms=float(t.item()))
        del eng
        dist.barrier()
    same = torch.equal(out["nccl"]["latent"], out["fused"]["latent"])
    a, b = out["nccl"]["latent"].double().flatten(), out["fused"]["latent"].double().flatten()
    rel = ((a - b).norm() / a.norm()).item()
    flags = torch.tensor([1 if same else 0], device=dev)
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(json.dumps({"selftest": "fused_vs_nccl", "world": world, "form": form.name, "bitwise_equal_all_ranks":
                          bool(flags.item()), "rel_l2": rel, "nccl_ms_per_step": round(out["nccl"]["ms"], 3),
                          "fused_ms_per_step": round(out["fused"]["ms"], 3), "model": cfg.name}))
        if args.record:
            from .autotune import record
            record(args.record, form.name, cfg.tokens(lat) // form.sp, out["nccl"]["ms"], out["fused"]["ms"],
                   bool(flags.item()), model=cfg.name, world=world)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
