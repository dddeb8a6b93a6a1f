"""Measure a B200 cost profile for the planner (ClusterCost JSON).

    python -m ditserve_b200.utils.calibrate --out profile.json                 # 1-GPU classes
    torchrun --nproc-per-node N -m ditserve_b200.utils.calibrate --merge profile.json --out profile.json

Single-GPU run: device-timed step of every video class at SP1 (both CFG branches), the
SD3.5 classes alone and as continuous batches (batch_step_ms) with their 2-D VAE decode,
and the Wan VAE decode.
Multi-GPU run: the step of each video class on the default CFG x Ulysses form of N GPUs
(fused path), merged into the class's measured ``forms`` table.  Forms that were not
measured are priced by the analytical model from step_compute_ms.  Random weights of the
real architectures, seeded synthetic inputs; max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

VIDEO = {
    "wan21_480p": dict(model="wan2.1-t2v-1.3b", height=480, width=832, frames=81, steps=50, heads=12),
    "wan22_720p": dict(model="wan2.2-ti2v-5b", height=704, width=1280, frames=121, steps=50, heads=24),
}
IMAGE = {"sd35_512": 512, "sd35_1024": 1024}


def _time(fn, iters=3, warmup=1, dev=None):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / iters
    if dist.is_initialized():
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def video_step(name, dev, layout=None, rank=0):
    from ..models.wan.config import CONFIGS
    from ..models.wan.runtime import WanEngine, WanSpec
    c = VIDEO[name]
    cfg = CONFIGS[c["model"]]
    spec = WanSpec(model=c["model"], height=c["height"], width=c["width"], frames=c["frames"], steps=c["steps"],
                   guidance=5.0, seed=1)
    pctx = plan = None
    if layout is not None:
        from ..parallel.runtime import build_parallel
        lat = spec.latent_shape()
        pctx, plan = build_parallel(layout, rank, dev, attention="fused", seq_local=cfg.tokens(lat) // layout.form.sp,
                                    cfg=cfg, pred_numel=lat[0] * lat[1] * lat[2] * lat[3])
    eng = WanEngine(cfg, device=dev, pctx=pctx, cfg_plan=plan, seed=0)
    st = eng.prepare(spec)
    ms = _time(lambda: eng.step(st), iters=3, warmup=2, dev=dev)
    del eng, st
    torch.cuda.empty_cache()
    return ms


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--merge", default=None)
    ap.add_argument("--classes", default=",".join(list(VIDEO) + list(IMAGE)))
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    wanted = args.classes.split(",")
    prof = json.load(open(args.merge)) if args.merge and os.path.exists(args.merge) else {
        "version": "ditserve-b200.profile.v1", "hardware": "B200 (sm_100a), NVLink 5 / NVSwitch",
        "sp_efficiency": {"2": 0.97, "3": 0.95, "4": 0.94, "6": 0.9, "8": 0.88},
        "links": {"default_gbps": 700.0, "default_latency_ms": 0.02},
        "quantum_overhead_ms": 2.0, "block_overhead_ms": 0.05, "resize_ms": 5.0, "sp_overlap": 0.3,
        "pair_overlap": 0.2, "classes": {}}
    classes = prof["classes"]
    if world == 1:
        for name in VIDEO:
            if name not in wanted:
                continue
            c = VIDEO[name]
            ms = video_step(name, dev)
            classes[name] = dict(kind="video", steps=c["steps"], blocks_per_step=30, heads=c["heads"],
                                 step_compute_ms=round(ms, 2), comm_mb_per_step=24200.0 if "21" in name else 40200.0,
                                 collectives_per_step=240, cfg_exchange_mb=4.2 if "21" in name else 10.5,
                                 forms={"sp1": {"step_ms": round(ms, 2)}})
            print(json.dumps({"class": name, "form": "sp1", "step_ms": round(ms, 2)}), flush=True)
        from ..models.sd35.model import SD35_MEDIUM
        from ..models.sd35.runtime import SD35Engine
        if any(n in wanted for n in IMAGE):
            eng = SD35Engine(SD35_MEDIUM, device=dev)
            for name, res in IMAGE.items():
                if name not in wanted:
                    continue
                table = {}
                for b in (1, 2, 4, 8):
                    sts = [eng.prepare(dict(height=res, width=res, steps=1000, seed=i)) for i in range(b)]
                    table[str(b)] = round(_time(lambda: eng.advance_batch(sts), iters=3, warmup=1), 2)
                from ..models.sd35.vae import SD35VAEDecoder
                if "vae" not in locals():
                    vae = SD35VAEDecoder.random_init(device=dev, dtype=torch.bfloat16, seed=1)
                zl = torch.randn(1, 16, res // 8, res // 8, device=dev, dtype=torch.bfloat16)
                decode = round(_time(lambda: vae.decode(zl), iters=3, warmup=1), 1)  # measured 2-D VAE decode
                classes[name] = dict(kind="image", steps=28, tokens=(res // 16) ** 2, step_ms=table["1"],
                                     service_ms=round(28 * table["1"] + decode, 1), decode_ms=decode,
                                     batch_step_ms=table)
                print(json.dumps({"class": name, "batch_step_ms": table}), flush=True)
            del eng
        if "wan21_480p" in classes:
            from ..models.wan.vae import WanVAEDecoder
            vae = WanVAEDecoder.random_init(device=dev, dtype=torch.bfloat16, seed=1)
            z = torch.randn(1, 16, 21, 60, 104, device=dev, dtype=torch.bfloat16)
            ms = _time(lambda: vae.decode(z), iters=1, warmup=1)
            classes["wan21_480p"]["decode_ms"] = round(ms, 1)
            classes["wan21_480p"]["decode_chunks"] = 4
            print(json.dumps({"class": "wan_vae_480p", "decode_ms": round(ms, 1)}), flush=True)
            del vae
            torch.cuda.empty_cache()
        if "wan22_720p" in classes:
            from ..models.wan.vae import WanVAEDecoder
            vae = WanVAEDecoder.random_init(device=dev, dtype=torch.bfloat16, seed=1, variant="wan2.2")
            z = torch.randn(1, 48, 31, 44, 80, device=dev, dtype=torch.bfloat16)  # 704x1280, 121 frames
            ms = _time(lambda: vae.decode(z), iters=1, warmup=1)
            classes["wan22_720p"]["decode_ms"] = round(ms, 1)
            classes["wan22_720p"]["decode_chunks"] = 4
            print(json.dumps({"class": "wan22_vae_720p", "decode_ms": round(ms, 1)}), flush=True)
            del vae
            torch.cuda.empty_cache()
    else:
        from ..parallel.layout import FixedLayout, default_form
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        form = default_form(world)
        layout = FixedLayout(tuple(range(world)), form)
        for name in VIDEO:
            if name not in wanted or name not in classes:
                continue
            if VIDEO[name]["heads"] % form.ulysses:
                continue
            ms = video_step(name, dev, layout, rank)
            classes[name].setdefault("forms", {})[form.name] = {"step_ms": round(ms, 2)}
            if rank == 0:
                print(json.dumps({"class": name, "form": form.name, "step_ms": round(ms, 2)}), flush=True)
        dist.destroy_process_group()
    if rank == 0:
        json.dump(prof, open(args.out, "w"), indent=1)


if __name__ == "__main__":
    main()
