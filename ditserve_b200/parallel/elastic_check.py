"""Multi-GPU check and timing of the elastic paths (doorbell group flag, regroup transfer).

    torchrun --nproc-per-node N -m ditserve_b200.parallel.elastic_check [--mb 40]

* group flag: ``GroupFlagPeer`` (one bounded-wait kernel) and ``GroupFlagNCCL`` (all_reduce
  MAX) agree on 64 random flag patterns; device-timed per-call latency of both;
* regroup transfer (SM stores and copy engines): a Wan-request-like snapshot (fp32 latents + solver history, ``--mb``
  MB in total) broadcast from rank 0 by ``PeerStateBroadcast`` and by
  ``broadcast_state_nccl``; both must be bit-identical to the source; device time of each
  (max over ranks);
* regroup latency with group formation: wall clock from "form a new group of ranks 0 and 1" to
  the first completed state transfer in it, for a peer-memory group and for a new NCCL group.
Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import time
from datetime import timedelta

import torch
import torch.distributed as dist


def _timed(fn, iters, dev):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mb", type=float, default=40.0)
    args = ap.parse_args()
    from .elastic import GroupFlagNCCL, GroupFlagPeer, PeerStateBroadcast, broadcast_state_nccl
    from .symm import SymmetricHeap
    rank, world, local = (int(os.environ[k]) for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    members = tuple(range(world))
    cap = int(args.mb * (1 << 20)) + (8 << 20)
    heap = SymmetricHeap(2 * cap + (8 << 20), dev)  # two broadcasters (the second for the new group)
    fp, fn = GroupFlagPeer(heap, members), GroupFlagNCCL(None, dev)
    g = torch.Generator().manual_seed(11)
    agree = True
    for _ in range(64):
        flags = torch.randint(0, 2, (world,), generator=g) * (torch.rand(world, generator=g) < 0.3)
        mine = int(flags[rank])
        agree &= fp(mine) == fn(mine) == int(flags.max())
    flag_peer_us = _timed(lambda: fp(0), 50, dev) * 1000
    flag_nccl_us = _timed(lambda: fn(0), 50, dev) * 1000

    n = int(args.mb * (1 << 20) / 4 / 5)
    n -= n % 4
    src = None
    if rank == 0:
        gen = torch.Generator(device=dev).manual_seed(5)
        src = dict(kind="wan_request.v1", step=3, latents=torch.randn(n, device=dev, generator=gen),
                   scheduler=dict(hist=[torch.randn(n, device=dev, generator=gen) for _ in range(3)],
                                  last=torch.randn(n + 3, device=dev, generator=gen), order=2))
    bc = PeerStateBroadcast(heap, members, cap)
    a = bc(src, 0)
    b = broadcast_state_nccl(src, 0, device=dev)
    ref = a if rank == 0 else None
    ok = all(torch.equal(x, y) for x, y in zip([a["latents"], *a["scheduler"]["hist"], a["scheduler"]["last"]],
                                               [b["latents"], *b["scheduler"]["hist"], b["scheduler"]["last"]]))
    ok &= a["step"] == 3 and a["scheduler"]["order"] == 2
    digest = torch.tensor([float(a["latents"].double().sum()), float(a["scheduler"]["last"].double().sum())],
                          device=dev, dtype=torch.float64)
    dg = [torch.zeros_like(digest) for _ in range(world)]
    dist.all_gather(dg, digest)
    ok &= all(torch.equal(d, dg[0]) for d in dg)
    # the same transfer by copy engines (one cudaMemcpyAsync per receiver and slice)
    bc.transport = "ce"
    c = bc(src, 0)
    ok_ce = all(torch.equal(x, y) for x, y in zip([a["latents"], *a["scheduler"]["hist"], a["scheduler"]["last"]],
                                                  [c["latents"], *c["scheduler"]["hist"], c["scheduler"]["last"]]))
    bc_ce_ms = _timed(lambda: bc(src, 0), 5, dev)
    bc.transport = "sm"
    bc_peer_ms = _timed(lambda: bc(src, 0), 5, dev)
    bc_nccl_ms = _timed(lambda: broadcast_state_nccl(src, 0, device=dev), 5, dev)
    nbytes = 4 * (4 * n + n + 3)
    # regroup latency including group formation (host wall clock to the first completed transfer,
    # max over ranks): a new peer-memory group is a host-side view of the existing heap, a new
    # NCCL group creates a communicator on its first collective
    sub = members[:2]
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    if rank in sub:
        bc2 = PeerStateBroadcast(heap, sub, int(args.mb * (1 << 20)) + (2 << 20), channel=8)
        bc2(src, 0)
        torch.cuda.synchronize()
    new_peer_ms = (time.perf_counter() - t0) * 1e3
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    pg = dist.new_group(list(sub))
    if rank in sub:
        broadcast_state_nccl(src, 0, device=dev, group=pg)
        torch.cuda.synchronize()
    new_nccl_ms = (time.perf_counter() - t0) * 1e3
    tt = torch.tensor([new_peer_ms, new_nccl_ms], device=dev, dtype=torch.float64)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    new_peer_ms, new_nccl_ms = (float(v) for v in tt.tolist())
    out = dict(world=world, flags_agree=bool(agree), flag_peer_us=round(flag_peer_us, 1),
               flag_nccl_us=round(flag_nccl_us, 1), state_mb=round(nbytes / 2 ** 20, 1), broadcast_bitwise=bool(ok),
               broadcast_peer_ms=round(bc_peer_ms, 3), broadcast_nccl_ms=round(bc_nccl_ms, 3),
               broadcast_ce_bitwise=bool(ok_ce), broadcast_ce_ms=round(bc_ce_ms, 3),
               broadcast_peer_gbs=round(nbytes * (world - 1) / bc_peer_ms / 1e6, 1),
               new_group_first_transfer_peer_ms=round(new_peer_ms, 2),
               new_group_first_transfer_nccl_ms=round(new_nccl_ms, 2))
    if rank == 0:
        print(json.dumps(out), flush=True)
    del ref
    dist.barrier()
    heap.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
