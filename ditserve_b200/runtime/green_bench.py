"""Co-located video and image work on one GPU, with and without a Green Context SM split.

    python -m ditserve_b200.runtime.green_bench [--video-sms 112] [--image-sms 36] [--steps 40]

A background thread keeps Wan2.1-1.3B DiT blocks (480p, both CFG branches) running on one
stream while the main thread runs SD3.5-Medium denoising steps (512x512, CFG batch of 2, 333
text tokens) one at a time on another stream; each image step is timed with CUDA events on its
own stream.  Two runs:

* ``shared``: plain streams, both workloads compete for all SMs;
* ``green``:  the video stream belongs to a green context with ``--video-sms`` SMs and the image
  stream to one with ``--image-sms`` SMs (``GreenPool``), so image steps never queue behind
  video kernels for SMs.

Printed: p50 / p99 / max image step latency for both runs, the video blocks completed meanwhile,
and an image-alone baseline on the full GPU.  Green contexts are a per-process view of the
device's SMs; nothing on the device is changed.  The CTA-pair GEMM is disabled here (its
two-SM clusters are placed by the partition's own rules), so both runs use the one-CTA GEMM.
Reference: workers/ditserve/runtime/green_context.py:64-269; results/5.7 of the reference
(image-step jitter 235.9 -> 4.2 ms with SM partitioning).
"""
from __future__ import annotations

import argparse
import json
import os
import threading

os.environ.setdefault("DS_GEMM_PAIR", "0")

import torch  # noqa: E402


def _pct(xs, q):
    xs = sorted(xs)
    return xs[min(len(xs) - 1, int(round(q * (len(xs) - 1))))]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--video-sms", type=int, default=112)
    ap.add_argument("--image-sms", type=int, default=36, help="the image role takes the SMs left after the video split")
    ap.add_argument("--steps", type=int, default=40)
    args = ap.parse_args(argv)
    from ..models.sd35.model import SD35_MEDIUM
    from ..models.sd35.runtime import SD35Engine
    from ..models.wan.config import WAN21_T2V_1_3B
    from ..models.wan.runtime import WanEngine, WanSpec
    from ..ops import check_status
    from .green_context import GreenPool

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    wan = WanEngine(WAN21_T2V_1_3B, device=dev, seed=0)
    img = SD35Engine(SD35_MEDIUM, device=dev)
    vstate = wan.prepare(WanSpec(model=WAN21_T2V_1_3B.name, height=480, width=832, frames=81, steps=1000,
                                 guidance=5.0, seed=1))
    istates = [img.prepare(dict(height=512, width=512, steps=100000, seed=2))]
    for _ in range(2):  # warm-up: allocator, tensor maps, weights layouts
        img.advance_batch(istates)
    wan.advance(vstate, blocks=2)
    torch.cuda.synchronize()

    def image_steps(stream):
        times = []
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                img.advance_batch(istates)
                e.record(stream)
                e.synchronize()
                times.append(s.elapsed_time(e))
        return times

    def run(video_stream, image_stream):
        stop = threading.Event()
        blocks = [0]

        def video():
            with torch.cuda.stream(video_stream):
                while not stop.is_set():
                    wan.advance(vstate, blocks=1)  # one DiT block (the last one also runs the step update)
                    video_stream.synchronize()
                    blocks[0] += 1
        th = threading.Thread(target=video, daemon=True)
        th.start()
        times = image_steps(image_stream)
        stop.set()
        th.join(timeout=120)
        torch.cuda.synchronize()
        return times, blocks[0]

    out = {}
    alone = image_steps(torch.cuda.Stream(dev))
    out["image_alone"] = dict(p50=round(_pct(alone, 0.5), 2), p99=round(_pct(alone, 0.99), 2))
    t, b = run(torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    out["shared"] = dict(p50=round(_pct(t, 0.5), 2), p99=round(_pct(t, 0.99), 2), max=round(max(t), 2),
                         video_blocks=b)
    pool = GreenPool(0, {"video": args.video_sms, "image": args.image_sms})
    try:
        t, b = run(pool.stream("video"), pool.stream("image"))
        out["green"] = dict(p50=round(_pct(t, 0.5), 2), p99=round(_pct(t, 0.99), 2), max=round(max(t), 2),
                            video_blocks=b, sm_counts=pool.sm_counts, total_sms=pool.total_sms)
    finally:
        torch.cuda.synchronize()
        pool.close()
    check_status(dev)
    out.update(image_steps=args.steps, image="sd3.5-medium 512x512 CFG batch 2",
               video="wan2.1-1.3b 480p CFG batch 2, one block per launch group", unit="ms per image step")
    print(json.dumps(out))


if __name__ == "__main__":
    main()
