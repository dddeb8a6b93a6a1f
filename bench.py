"""Headline benchmark: per-step DiT latency of the Wan2.1-T2V-1.3B-shaped model.

Config (second config): bf16, random init, 30 blocks, dim 1536,
12 heads x 128, FFN 8960, 480x832x81 video -> latent 16x21x60x104 -> 32 760
tokens, 512x4096 text context drawn N(0, 1), UniPC flow solver, CFG 5.0.
One "step" = both CFG branches of the DiT + the fused CFG/UniPC update.

Parallel form by GPU count (strong scaling: the same request on more GPUs):
    N=1 sp1 (both branches batched), N=2 cfg2, N=4 cfg2sp2, N=8 cfg2sp4.

    python bench.py [--gpus N --steps K --warmup W]          # our engine
    python bench.py --impl reference ...                       # the reference's own stack

Timing: W untimed warm-up steps; then K steps bracketed by a barrier and
torch.cuda.synchronize, timed with CUDA events on the launching stream; the
max over ranks is reported.  Activations (0.2-1.2 GB per step) exceed the
126 MB L2, so no explicit flush is needed between steps.  The end-to-end
figure repeats the measurement through the public engine API with the step's
inputs (latent + text embeddings) copied from pinned host memory and the new
latent read back every step.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# published per-step latency of the reference for this request class (Wan2.1 480p tier,
# 32 760 tokens; results/5.1_Experimental_Setup/README.md:33-34 of the reference):
# SP1 on 1x A100 and CFG2 on 2x A100.
PUBLISHED_MS = {1: 3965.0, 2: 1998.0}
METRIC = "wan2.1-1.3b 480p (32760 tok) DiT step latency, CFG 5.0"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--attention", choices=["fused", "nccl"], default="fused")
    ap.add_argument("--no-e2e", action="store_true")
    return ap.parse_args()


class ClockSampler:
    """nvidia-smi clock/throttle samples taken while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(",") for r in out.strip().splitlines() if r.strip()]
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


def reference_arm(args):
    """Run the unmodified reference through its own public API, or say why it cannot run.

    The reference's Wan entry point is ``ditserve.models.wan.runtime.WanStepWorker``
    (installed from the reference tree into baseline/_ref).  The probe walks the
    path a user of the reference takes, in order, and reports the first step that
    fails with the exception text verbatim: the install is present, ``import
    ditserve`` works, the worker module imports, and the worker constructs on this
    rank's GPU.  When the constructor fails, the packages it pins are then looked up
    (installed version or "not installed") and listed after the failure as facts of
    this box, not as the cause.
    """
    import importlib
    import importlib.metadata as md

    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    def unavailable(reason: str) -> int:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": reason}))
        return 0

    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "ditserve")):
        return unavailable(f"the reference is not installed on this box: {ref}/ditserve does not exist")
    sys.path.insert(0, ref)
    try:
        importlib.import_module("ditserve")
    except Exception as exc:
        return unavailable(f"import ditserve (from {ref}) failed: {type(exc).__name__}: {exc}")
    try:
        runtime = importlib.import_module("ditserve.models.wan.runtime")
    except Exception as exc:
        return unavailable(f"import ditserve.models.wan.runtime failed: {type(exc).__name__}: {exc}")
    try:
        runtime.WanStepWorker(device=f"cuda:{local}", attention="flash")
    except Exception as exc:
        facts = []
        for pkg, want in getattr(runtime, "REQUIRED_VERSIONS", {}).items():
            try:
                have = md.version(pkg)
            except md.PackageNotFoundError:
                have = "not installed"
            facts.append(f"{pkg}: pinned {want}, here {have}")
        tail = f" [{'; '.join(facts)}]" if facts else ""
        return unavailable(f"WanStepWorker(device='cuda:{local}', attention='flash') raised "
                           f"{type(exc).__name__}: {exc}{tail}")
    return unavailable("WanStepWorker constructed, but bench.py has no offline Wan snapshot for it to serve")


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    import torch
    import torch.distributed as dist

    from ditserve_b200 import ops
    from ditserve_b200.models.wan.config import WAN21_T2V_1_3B
    from ditserve_b200.models.wan.model import LocalAttention
    from ditserve_b200.models.wan.runtime import CFGLocal, WanEngine, WanSpec
    from ditserve_b200.parallel.layout import FixedLayout, default_form

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    form = default_form(world)
    pctx, cfg_plan = LocalAttention(), CFGLocal()
    layout = FixedLayout(tuple(range(world)), form)
    nccl_plans = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        from ditserve_b200.parallel.runtime import build_parallel
        kw = dict(seq_local=WAN21_T2V_1_3B.tokens((16, 21, 60, 104)) // form.sp, cfg=WAN21_T2V_1_3B,
                  pred_numel=16 * 21 * 60 * 104)
        pctx, cfg_plan = build_parallel(layout, rank, dev, attention=args.attention, **kw)
        if args.attention == "fused":
            nccl_plans = build_parallel(layout, rank, dev, attention="nccl", **kw)

    engine = WanEngine(WAN21_T2V_1_3B, device=dev, pctx=pctx, cfg_plan=cfg_plan, seed=0)
    spec = WanSpec(model=WAN21_T2V_1_3B.name, height=480, width=832, frames=81, steps=50, guidance=5.0, seed=42)

    def set_plans(plans):
        engine.pctx, engine.cfg_plan = plans

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    st = engine.prepare(spec)
    check = None
    if nccl_plans is not None:
        # Untimed check before warm-up: one step of the same state through the NCCL path and
        # through the fused peer-memory path; the latents must agree bit for bit on every rank.
        snap = engine.snapshot(st, device=dev)
        fused_plans = (engine.pctx, engine.cfg_plan)
        set_plans(nccl_plans)
        st_n = engine.step(engine.restore(snap))
        set_plans(fused_plans)
        st_f = engine.step(engine.restore(snap))
        torch.cuda.synchronize()
        a, b = st_n.latents.double().flatten(), st_f.latents.double().flatten()
        flags = torch.tensor([1.0 if torch.equal(st_n.latents, st_f.latents) else 0.0,
                              -((a - b).norm() / a.norm()).item()], device=dev, dtype=torch.float64)
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
        check = {"fused_equals_nccl": bool(flags[0].item() == 1.0), "max_rel_l2": float(-flags[1].item()),
                 "compared": "latents after one step from the same state, all ranks"}
        del st_n, st_f, snap
    for _ in range(args.warmup):
        engine.step(st)
    torch.cuda.synchronize()
    ops.check_status(dev)
    ops.launch_counts(reset=True)

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("ds_step")
    t0.record()
    for _ in range(args.steps):
        if st.done:
            raise SystemExit("increase the schedule length")
        engine.step(st)
    t1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    launches = sum(ops.launch_counts(reset=True).values())
    ms = max_over_ranks(t0.elapsed_time(t1) / args.steps)
    ops.check_status(dev)

    # per-kernel device time of one more (untimed) step: CUDA events around every launch of
    # this package's kernels on the launching stream, summed per entry point, max over ranks
    breakdown = None
    if not st.done:
        with ops.KernelTimer() as kt:
            b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            b0.record()
            engine.step(st)
            b1.record()
            totals = kt.totals_ms()
        names = sorted(set(totals) | {"gemm", "attention", "attention_scatter", "qkv_scatter", "group_barrier",
                                      "allgather_rows", "cfg_step_peer", "layernorm_modulate", "rmsnorm_rope",
                                      "sched_step"})
        vec = torch.tensor([totals.get(n, 0.0) for n in names] + [b0.elapsed_time(b1)], device=dev,
                           dtype=torch.float64)
        if world > 1:
            dist.all_reduce(vec, op=dist.ReduceOp.MAX)
        vals = vec.tolist()
        step_ms = vals[-1]
        per_kernel = {n: round(v, 3) for n, v in zip(names, vals[:-1]) if v > 0}
        breakdown = {"step_ms": round(step_ms, 3), "kernels_ms": per_kernel,
                     "outside_kernels_ms": round(step_ms - sum(vals[:-1]), 3),
                     "how": "one untimed step with CUDA events around each launch (adds host work per launch); "
                            "max over ranks per entry"}
    ops.check_status(dev)

    e2e = None
    if not args.no_e2e:
        # end to end through the public API: inputs from pinned host memory, result read back
        st2 = engine.prepare(spec)
        host_lat = st2.latents.cpu().pin_memory()
        host_ctx = st2.context.cpu().pin_memory()
        host_neg = st2.negative.cpu().pin_memory()
        out_host = torch.empty_like(host_lat).pin_memory()
        for _ in range(2):
            engine.step(st2)
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            st2.latents.copy_(host_lat, non_blocking=True)
            st2.context.copy_(host_ctx, non_blocking=True)
            st2.negative.copy_(host_neg, non_blocking=True)
            engine.step(st2)
            out_host.copy_(st2.latents, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        h2d = host_lat.numel() * host_lat.element_size() + 2 * host_ctx.numel() * host_ctx.element_size()
        e2e = {"value": round(e2e_ms, 3), "unit": "ms/step", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(out_host.numel() * out_host.element_size())}

    if rank == 0:
        pub = PUBLISHED_MS.get(world)
        line = {
            "metric": METRIC, "value": round(ms, 3), "unit": "ms/step", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None if pub is None else round(ms / pub, 4), "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) latent and text embeddings, random-init weights)",
            "config": {"model": "wan2.1-t2v-1.3b-shaped DiT (30 blocks, dim 1536, 12x128 heads, FFN 8960)",
                       "global_batch": 1, "seq_len": 32760, "text_len": 512, "cfg": 5.0,
                       "parallelism": form.name, "attention_path": "local" if world == 1 else args.attention,
                       "l2": "no flush: per-step activations (0.2-1.2 GB) exceed the 126 MB L2"},
            "clocks": clk, "e2e": e2e, "gpu_launches": launches,
        }
        if check is not None:
            line.update(check)
        if breakdown is not None:
            line["breakdown"] = breakdown
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
