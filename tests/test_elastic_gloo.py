"""Elastic layout pieces on CPU: epoch guard, reshard codec, lockstep pairs, and the
consensus / group flag / regroup broadcast paths as 2-rank gloo worlds."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ditserve_b200.parallel.elastic import (LayoutHandle, StaleLayout, merge_tokens, reshard, split_tokens)
from ditserve_b200.parallel.layout import FixedLayout, Form


def test_layout_handle_epochs():
    h = LayoutHandle()
    a = FixedLayout((0, 1), Form.parse("sp2"), 1)
    h.propose(a)
    with pytest.raises(StaleLayout):
        h.activate(False)
    h.activate(True)
    h.check(1)
    with pytest.raises(StaleLayout):
        h.check(0)
    with pytest.raises(StaleLayout):
        h.propose(FixedLayout((0, 1), Form.parse("cfg2"), 1))


def test_reshard_exact():
    x = torch.randn(2, 1001, 8)
    s2, pad = split_tokens(x, 2)
    assert torch.equal(merge_tokens(s2, pad), x)
    s6, pad6 = reshard(s2, pad, 6)
    assert len(s6) == 6 and torch.equal(merge_tokens(s6, pad6), x)


def test_advance_pair_matches_single():
    from ditserve_b200.models.wan.runtime import WanEngine
    e = WanEngine("wan-tiny", device="cpu", dtype=torch.float32)
    spec = dict(model="wan-tiny", height=64, width=64, frames=5, steps=2)
    a, b = e.prepare(dict(spec, seed=1)), e.prepare(dict(spec, seed=2))
    a2, b2 = e.prepare(dict(spec, seed=1)), e.prepare(dict(spec, seed=2))
    r = e.advance_pair(a, b, 1)
    assert r["a"]["next_block"] == 1 and not r["a"]["step_completed"]
    r = e.advance_pair(a, b)
    assert r["a"]["step_completed"] and r["b"]["step_completed"]
    e.step(a2)
    e.step(b2)
    assert torch.equal(a.latents, a2.latents) and torch.equal(b.latents, b2.latents)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, tmp, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ditserve_b200.models.wan.backend import WanBackend
        from ditserve_b200.parallel.elastic import GroupFlagNCCL, RequestGroupGate
        w = WanBackend({"model": "wan-tiny", "device": "cpu", "transfer_dir": tmp})
        spec = dict(request_id="r", height=64, width=64, frames=5, steps=2, seed=7)
        if rank == 0:
            w.prepare(dict(id=1, spec=spec))
            w.advance(dict(id=2, state_id="r", steps=1))
        # regroup: rank 1 joins the request (NCCL-path broadcast, gloo here)
        out = w.distributed(dict(id=3, action="migrate_group", ranks=[0, 1], src=0, state_id="r", path="nccl"))
        assert out["step"] == 1
        c = w.distributed(dict(id=4, action="consensus", ranks=[0, 1], state_id="r", epoch=1))
        flag = GroupFlagNCCL(None, "cpu")(rank)  # MAX over {0, 1}
        # divergence: rank 1 advances one more step, consensus must fail
        w.advance(dict(id=5, state_id="r", steps=1)) if rank == 1 else None
        bad = RequestGroupGate(None).consensus(str(w.states["r"].step))
        q.put((rank, c["agreed"], flag, bad, w.states["r"].latents.sum().item()))
    finally:
        dist.destroy_process_group()


def test_regroup_consensus_flag_gloo(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path), q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(240)
    assert all(p.exitcode == 0 for p in ps)
    res = sorted(q.get() for _ in range(2))
    assert res[0][1] and res[1][1]          # agreed after the regroup
    assert res[0][2] == 1 and res[1][2] == 1  # MAX flag
    assert not res[0][3] and not res[1][3]    # divergence detected


def test_collective_autotune_table(tmp_path):
    from ditserve_b200.parallel.autotune import choose, load, record
    t = tmp_path / "c.json"
    record(t, "cfg2sp4", 9408, nccl_ms=2.19, fused_ms=1.70, bitwise=True)
    record(t, "cfg2u2r2", 9408, nccl_ms=2.38, fused_ms=2.48, bitwise=False)
    record(t, "cfg2u2r2", 1 << 20, nccl_ms=90.0, fused_ms=80.0, bitwise=False)
    e = load(t)
    assert len(e) == 3
    assert choose("cfg2sp4", 10000, e) == "fused"
    assert choose("cfg2u2r2", 9000, e) == "nccl" and choose("cfg2u2r2", 900000, e) == "fused"
    assert choose("sp2", 100, e) == "fused"  # never measured: default
