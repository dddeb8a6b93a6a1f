"""FP8 payloads for the Ulysses all-to-alls (NCCL path): codec bounds, a Gloo SP2 run of the
tiny Wan DiT against the bf16 path, per-block calibration and the bytes on the wire."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ditserve_b200.parallel.fp8_comms import E4M3_MAX, fp8_pack, fp8_unpack, payload_bytes


def test_codec_round_trip_bound():
    torch.manual_seed(0)
    x = torch.randn(257, 128) * torch.logspace(-3, 3, 257)[:, None]
    buf = fp8_pack(x)
    assert buf.dtype == torch.uint8 and buf.shape == (257, 132)
    y = fp8_unpack(buf, 128, torch.float32)
    # e4m3 keeps 3 mantissa bits: per element |err| <= 2^-4 |x| above the subnormal range,
    # and within half a subnormal step (2^-10 of the row scale) below it
    scale = x.abs().amax(dim=1, keepdim=True) / E4M3_MAX
    assert ((y - x).abs() <= torch.maximum(x.abs() / 16, scale * 2.0 ** -10) + 1e-30).all()
    assert fp8_unpack(fp8_pack(torch.zeros(3, 8)), 8, torch.float32).abs().max() == 0
    assert payload_bytes(10, 128, True) / payload_bytes(10, 128, False) == pytest.approx(132 / 256)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


SPEC = dict(model="wan-tiny", height=64, width=64, frames=13, steps=3, guidance=5.0, seed=7)


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ditserve_b200.models.wan.config import WAN_TINY
        from ditserve_b200.models.wan.runtime import WanEngine
        from ditserve_b200.parallel.fp8_comms import calibrate
        from ditserve_b200.parallel.layout import FixedLayout, Form
        from ditserve_b200.parallel.runtime import build_parallel
        layout = FixedLayout((0, 1), Form(1, 2, 1))
        res = {}
        for path in ("nccl", "nccl-fp8"):
            pctx, cfg_plan = build_parallel(layout, rank, torch.device("cpu"), attention=path)
            torch.manual_seed(0)
            e = WanEngine(WAN_TINY, device="cpu", dtype=torch.float32, pctx=pctx, cfg_plan=cfg_plan, seed=1)
            st = e.prepare(SPEC)
            e.run(st)
            res[path] = (st.latents.clone(), getattr(pctx, "bytes_sent", None))
        # calibration on one probe packet: a loose bound keeps every block, a zero bound none
        pctx, cfg_plan = build_parallel(layout, rank, torch.device("cpu"), attention="nccl-fp8")
        torch.manual_seed(0)
        e = WanEngine(WAN_TINY, device="cpu", dtype=torch.float32, pctx=pctx, cfg_plan=cfg_plan, seed=1)
        st = e.prepare(SPEC)
        _, lat, t, ctx = e._inputs(st)
        with torch.inference_mode():
            pk = e.model.begin(lat, t, ctx, pctx)
            cal_loose = calibrate(e.model, pk, pctx, max_rel_error=0.5)
            cal_zero = calibrate(e.model, pk, pctx, max_rel_error=0.0)
        if rank == 0:
            out["bf16"], _ = res["nccl"]
            out["fp8"], out["fp8_bytes"] = res["nccl-fp8"]
            out["cal_loose"], out["cal_zero"] = cal_loose, cal_zero
    finally:
        dist.destroy_process_group()


def test_fp8_sp2_gloo_matches_bf16_and_calibrates():
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
    a, b = out["bf16"].double().flatten(), out["fp8"].double().flatten()
    cos = float(torch.dot(a, b) / (a.norm() * b.norm()))
    rel = float((a - b).norm() / a.norm())
    assert cos >= 0.99 and rel <= 0.1, (cos, rel)
    assert out["fp8_bytes"] > 0
    assert out["cal_loose"]["layers"] == [0, 1]
    assert out["cal_zero"]["layers"] == []
    assert all(0 < v < 0.5 for v in out["cal_loose"]["errors"].values())
