"""INT8 ring key/value codec: arithmetic, anchor schedule, the NCCL-path transport on a Gloo
world of 4 (Ulysses 2 x ring 2) against the bf16 ring under the bounded-drift gate, and the
fused-path kernels (ring_quant_push / ring_dequant) against the torch statement on one GPU."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ditserve_b200.parallel.ring_codec import RingInt8Codec, make_codec


def test_codec_round_trip_and_bytes():
    g = torch.Generator().manual_seed(0)
    x = (torch.randn(64, 12 * 128, generator=g) * torch.rand(64, 1, generator=g) * 4).bfloat16()
    q, s = RingInt8Codec.encode(x, 128)
    assert q.dtype == torch.int8 and s.dtype == torch.float32 and s.shape == (64, 12)
    assert int(q.abs().max()) == 127  # every vector uses the full range
    y = RingInt8Codec.decode(q, s, 128)
    err = (y.float() - x.float()).abs().reshape(64, 12, 128)
    assert torch.all(err <= s[..., None] * 0.5 + x.float().abs().reshape(64, 12, 128) * 2 ** -8 + 1e-6)
    cos = torch.nn.functional.cosine_similarity(x.float().flatten(), y.float().flatten(), dim=0)
    assert cos > 0.999
    assert RingInt8Codec.wire_bytes(1, 1, 128, True) == 2 * 132
    assert RingInt8Codec.wire_bytes(1, 1, 128, False) == 2 * 256
    z = torch.zeros(4, 256).bfloat16()
    qz, sz = RingInt8Codec.encode(z, 128)
    assert torch.equal(RingInt8Codec.decode(qz, sz, 128), z)


def test_anchor_schedule():
    c = RingInt8Codec(warmup_steps=2, tail_anchor_steps=2)
    assert [c.should_quantize(i, 10) for i in range(10)] == [False, False] + [True] * 6 + [False, False]
    assert not RingInt8Codec(enabled=False).should_quantize(5, 10)
    assert make_codec(None) is None and make_codec("off") is None
    assert make_codec("int8").warmup_steps == 2
    assert make_codec({"warmup_steps": 1, "tail_anchor_steps": 0}).should_quantize(9, 10)
    with pytest.raises(ValueError):
        make_codec("fp4")


SPEC = dict(model="wan-tiny", height=64, width=64, frames=13, steps=4, guidance=5.0, seed=7)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ditserve_b200.models.wan.config import WAN_TINY
        from ditserve_b200.models.wan.runtime import WanEngine
        from ditserve_b200.parallel.layout import FixedLayout, Form
        from ditserve_b200.parallel.runtime import build_parallel
        layout = FixedLayout(tuple(range(world)), Form(1, 4, 2))
        results = {}
        for name, codec in (("bf16", None), ("int8", {"warmup_steps": 1, "tail_anchor_steps": 1})):
            pctx, plan = build_parallel(layout, rank, torch.device("cpu"), attention="nccl", ring_codec=codec)
            torch.manual_seed(0)
            e = WanEngine(WAN_TINY, device="cpu", dtype=torch.float32, pctx=pctx, cfg_plan=plan, seed=1)
            st = e.run(e.prepare(SPEC))
            results[name] = st.latents.clone()
            if codec is not None:
                results["stats"] = pctx.codec.summary()
        if rank == 0:
            out.update(results)
    finally:
        dist.destroy_process_group()


def test_int8_ring_on_gloo_u2r2_stays_within_the_drift_gate():
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(4, port, out), nprocs=4, join=True)
    a, b = out["bf16"].flatten().double(), out["int8"].flatten().double()
    cos = (torch.dot(a, b) / (a.norm() * b.norm())).item()
    rel = ((a - b).norm() / a.norm()).item()
    assert cos >= 0.95 and rel <= 0.25, (cos, rel)
    assert not torch.equal(out["bf16"], out["int8"])  # the codec really ran on the middle steps
    stats = out["stats"]
    # 4 steps x 2 blocks, one peer chunk each: steps 1 and 2 int8, steps 0 and 3 bf16 anchors
    assert stats["int8_chunks"] == 4 and stats["bf16_chunks"] == 4, stats


@pytest.mark.gpu
@pytest.mark.parametrize("hd,heads", [(128, 6), (64, 8)])
def test_ring_kernels_match_the_torch_statement(hd, heads):
    from ditserve_b200 import ops
    ext = ops.ext()
    dev = torch.device("cuda", 0)
    rows = 1000
    w = heads * hd
    g = torch.Generator(device=dev).manual_seed(hd)
    recv = (torch.randn(rows, 3 * w, device=dev, generator=g) * 3).bfloat16()
    slot = int(ext.ring_slot_bytes(rows, heads, hd))
    flag = max(65536, int(ext.FLAG_BYTES))
    heap, _ = ext.symm_alloc(flag + 2 * slot + 4096, 0)
    base = heap.data_ptr()
    # a two-member "ring" whose members share one heap: rank 0 pushes its packet into slot 0
    # of member 1 (this heap), then member 1 decodes slot 0 locally
    ext.ring_quant_push(recv[:, w:], heads, hd, 0, flag, slot, 0, [base, base], int(1e9))
    out = torch.zeros(rows, 3 * w, device=dev, dtype=torch.bfloat16)
    ext.ring_dequant(out, heads, hd, 0, flag, slot, 1, [base, base], int(1e9))
    torch.cuda.synchronize()
    q8, sc = RingInt8Codec.encode(recv[:, w:].cpu(), hd)
    got_q = heap[flag:flag + rows * 2 * w].view(torch.int8).view(rows, 2 * w).cpu()
    got_s = heap[flag + rows * 2 * w:flag + rows * 2 * w + rows * 2 * heads * 4].view(torch.float32)
    assert torch.equal(got_q, q8)
    assert torch.equal(got_s.view(rows, 2 * heads).cpu(), sc)
    assert torch.equal(out[:, w:].cpu(), RingInt8Codec.decode(q8, sc, hd))
    assert int(out[:, :w].abs().sum()) == 0  # the q columns of the decoded buffer are not written
