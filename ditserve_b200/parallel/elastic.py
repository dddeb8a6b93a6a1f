"""Elastic layouts: epoch guard, step-boundary consensus, reshard codec, regroup transfer.

* ``LayoutHandle`` — the active ``FixedLayout`` of a worker with a monotonically increasing
  epoch.  A new layout is staged with ``propose`` and becomes active only through
  ``activate`` at a solver-step boundary; messages carrying another epoch are rejected
  (reference: LayoutHandle, workers/ditserve/models/wan/parallel.py:173-254).
* ``RequestGroupGate`` — all ranks of a group agree on (request, step, block, epoch and a
  device checksum of the latents) before a layout change or a step commit: one
  ``all_gather_object`` of a digest (reference: RequestGroupGate.consensus, parallel.py:296-365).
* ``split_tokens`` / ``merge_tokens`` / ``reshard`` — exact split of a token sequence into
  SP shards and back, and re-sharding between SP degrees (reference: parallel.py:579-618).
* Doorbell group flag (MAX of a stop flag over an SP group): ``GroupFlagNCCL`` is the
  all_reduce baseline, ``GroupFlagPeer`` one bounded-wait kernel over peer memory.
* Regroup state transfer (a request's latents and solver history reach the ranks that join
  its new group): ``broadcast_state_nccl`` is the per-tensor NCCL broadcast baseline,
  ``PeerStateBroadcast`` stores every tensor straight into the joining ranks' heaps with
  multi-peer put kernels: small tensors go to every receiver directly, large ones as a
  scatter (slice j to receiver j) followed by an all-gather among the receivers, so the
  source's NVLink egress carries each byte once; bounded barriers between phases; bit-exact (reference: CacheOffGroupMigration,
  parallel.py:903-1050; host-staged packet files, study.cpp:1395-1411).
"""
from __future__ import annotations

import hashlib
import json
import math

import torch
import torch.distributed as dist


class StaleLayout(RuntimeError):
    pass


class LayoutHandle:
    def __init__(self):
        self.layout = None
        self.epoch = -1
        self.pending = None

    def propose(self, layout):
        if layout.epoch <= self.epoch or (self.pending is not None and layout.epoch <= self.pending.epoch):
            raise StaleLayout(f"layout epoch {layout.epoch} is not newer than {max(self.epoch, getattr(self.pending, 'epoch', -1))}")
        self.pending = layout

    def activate(self, at_step_boundary: bool):
        if self.pending is None:
            raise StaleLayout("no layout proposed")
        if not at_step_boundary:
            raise StaleLayout("a layout may change only at a solver-step boundary")
        self.layout, self.epoch, self.pending = self.pending, self.pending.epoch, None
        return self.layout

    def check(self, epoch: int):
        if epoch != self.epoch:
            raise StaleLayout(f"message for layout epoch {epoch}, active epoch is {self.epoch}")


def state_digest(state_id: str, st, epoch: int) -> str:
    """Digest of a request's position plus a device checksum of its latents (no values leave the GPU)."""
    lat = st.latents
    chk = int(lat.detach().contiguous().view(torch.int32).to(torch.int64).sum().item()) if lat.element_size() == 4 \
        else float(lat.double().sum().item())
    body = dict(id=state_id, step=int(st.step), block=int(st.block), epoch=int(epoch), checksum=chk)
    return hashlib.sha256(json.dumps(body, sort_keys=True).encode()).hexdigest()


class RequestGroupGate:
    def __init__(self, group=None):
        self.group = group

    def consensus(self, digest: str) -> bool:
        n = dist.get_world_size(self.group)
        got = [None] * n
        dist.all_gather_object(got, digest, group=self.group)
        return all(g == digest for g in got)


def split_tokens(x: torch.Tensor, parts: int, dim: int = 1):
    """Split along ``dim`` into ``parts`` equal shards, zero-padding the tail; returns (shards, pad)."""
    n = x.shape[dim]
    per = math.ceil(n / parts)
    pad = per * parts - n
    if pad:
        shape = list(x.shape)
        shape[dim] = pad
        x = torch.cat([x, x.new_zeros(shape)], dim)
    return list(x.split(per, dim)), pad


def merge_tokens(shards, pad: int = 0, dim: int = 1) -> torch.Tensor:
    x = torch.cat(list(shards), dim)
    return x.narrow(dim, 0, x.shape[dim] - pad) if pad else x


def reshard(shards, pad: int, new_parts: int, dim: int = 1):
    return split_tokens(merge_tokens(shards, pad, dim), new_parts, dim)


class GroupFlagNCCL:
    def __init__(self, group, device):
        self.group = group
        self.buf = torch.zeros(1, dtype=torch.int32, device=device)

    def __call__(self, flag: int) -> int:
        self.buf.fill_(int(flag))
        dist.all_reduce(self.buf, op=dist.ReduceOp.MAX, group=self.group)
        return int(self.buf.item())


class GroupFlagPeer:
    """MAX of a 0/1 flag over a peer group in one launch (two alternating channels)."""

    def __init__(self, heap, members: tuple, channels=(5, 6), timeout_s: float = 10.0):
        from ..ops._ext import ext
        from .symm import PeerGroup
        self.ext = ext()
        self.groups = [PeerGroup(heap, members, c, timeout_s) for c in channels]
        self.heap = heap
        self.count = 0
        self.out = torch.zeros(1, dtype=torch.int32, device=heap.device)

    def __call__(self, flag: int) -> int:
        from ..ops._ext import check_status, status_word
        g = self.groups[self.count % 2]
        self.count += 1
        self.ext.group_flag(g.rank, g.bases, g.timeout_ns, g.channel, self.heap.next_epoch(g.channel), int(bool(flag)),
                            self.out, status_word(self.heap.device))
        v = int(self.out.item())
        check_status(self.heap.device)
        return v


def _tensors(tree, out):
    if isinstance(tree, torch.Tensor):
        out.append(tree)
        return ("__tensor__", len(out) - 1, list(tree.shape), str(tree.dtype).replace("torch.", ""))
    if isinstance(tree, dict):
        return {k: _tensors(v, out) for k, v in tree.items()}
    if isinstance(tree, (list, tuple)):
        return [_tensors(v, out) for v in tree]
    return tree


def _rebuild(desc, tensors):
    if isinstance(desc, (list, tuple)) and len(desc) == 4 and desc[0] == "__tensor__":
        return tensors[desc[1]]
    if isinstance(desc, dict):
        return {k: _rebuild(v, tensors) for k, v in desc.items()}
    if isinstance(desc, list):
        return [_rebuild(v, tensors) for v in desc]
    return desc


def _specs(desc, out):
    if isinstance(desc, (list, tuple)) and len(desc) == 4 and desc[0] == "__tensor__":
        out.append((desc[2], getattr(torch, desc[3])))
    elif isinstance(desc, dict):
        for v in desc.values():
            _specs(v, out)
    elif isinstance(desc, list):
        for v in desc:
            _specs(v, out)
    return out


def broadcast_state_nccl(tree, src: int, group=None, device=None):
    """Broadcast a nested dict of tensors (a request snapshot) from global rank ``src``."""
    me = dist.get_rank()
    tensors = []
    desc = _tensors(tree, tensors) if me == src else None
    box = [desc]
    dist.broadcast_object_list(box, src=src, group=group)
    desc = box[0]
    if me == src:
        out = [t.contiguous() for t in tensors]
    else:
        out = [torch.empty(shape, dtype=dt, device=device) for shape, dt in _specs(desc, [])]
    for t in out:
        dist.broadcast(t, src=src, group=group)
    return _rebuild(desc, out)


class PeerStateBroadcast:
    """Regroup transfer over peer memory: the source puts every tensor into the receivers' heaps.

    ``transport="sm"`` stores with the ``put_peers`` kernel (16-byte NVLink stores from SMs);
    ``transport="ce"`` issues one ``cudaMemcpyAsync`` per receiver and slice on the current
    stream, so the copy engines move the bytes and the SMs stay free for compute.  Both are
    ordered before the group barrier that publishes the data (reference copy-engine path:
    workers/gfc/kernels/copy_engine.py:21-133)."""

    def __init__(self, heap, members: tuple, capacity_bytes: int, channel: int = 7, timeout_s: float = 10.0,
                 group=None, transport: str = "sm"):
        from ..ops._ext import ext
        from .symm import PeerGroup
        self.ext = ext()
        self.group = PeerGroup(heap, members, channel, timeout_s)
        self.pg = group
        self.heap = heap
        self.capacity = int(capacity_bytes)
        self.off = heap.alloc(self.capacity, align=4096)
        self.scatter_min_bytes = 1 << 20  # larger tensors go scatter + all-gather (bandwidth-optimal)
        if transport not in ("sm", "ce"):
            raise ValueError("transport must be sm or ce")
        self.transport = transport

    def _put(self, src: torch.Tensor, mask: int, dst_off: int, r, bases, tmo):
        if self.transport == "sm":
            self.ext.put_peers(src, mask, dst_off, r, bases, tmo)
            return
        from cuda.bindings import runtime as cudart
        stream = torch.cuda.current_stream(src.device).cuda_stream
        nbytes = src.numel() * src.element_size()
        for m, base in enumerate(bases):
            if mask >> m & 1:
                err, = cudart.cudaMemcpyAsync(base + dst_off, src.data_ptr(), nbytes,
                                              cudart.cudaMemcpyKind.cudaMemcpyDefault, stream)
                if err != cudart.cudaError_t.cudaSuccess:
                    raise RuntimeError(f"copy-engine put to member {m} failed: {err}")

    def __call__(self, tree, src_member: int, src_global: int | None = None):
        """``src_member`` indexes the group; ``src_global`` is its rank in the default group
        (defaults to the member's heap rank, which is the global rank for a world heap)."""
        from ..ops._ext import check_status, status_word
        g = self.group
        status = status_word(self.heap.device)
        src_global = g.members[src_member] if src_global is None else src_global
        tensors = []
        desc = _tensors(tree, tensors) if g.rank == src_member else None
        box = [desc]
        dist.broadcast_object_list(box, src=src_global, group=self.pg)
        desc = box[0]
        specs = _specs(desc, [])
        offs, cur = [], 0
        for shape, dt in specs:
            nb = math.prod(shape) * torch.empty((), dtype=dt).element_size()
            offs.append(cur)
            cur += (nb + 4095) // 4096 * 4096
        if cur > self.capacity:
            raise MemoryError(f"state of {cur} bytes exceeds the broadcast staging area ({self.capacity})")
        r, bases, tmo = g.args()
        receivers = [m for m in range(g.size) if m != src_member]
        k = len(receivers)
        sizes = [math.prod(shape) * torch.empty((), dtype=dt).element_size() for shape, dt in specs]

        def split(nb):
            """16-byte-aligned slice bounds of the scattered body (one slice per receiver)."""
            body = nb // 16 * 16
            if k < 2 or body < self.scatter_min_bytes:
                return body, None
            per = -(-body // 16 // k) * 16
            return body, [(j * per, min(body, (j + 1) * per)) for j in range(k)]

        if g.rank == src_member:
            everyone = ((1 << g.size) - 1) & ~(1 << src_member)
            for t, o, nb in zip(tensors, offs, sizes):
                flat = t.contiguous().view(-1).view(torch.uint8)
                body, parts = split(nb)
                if parts is None:  # small: store the whole body into every receiver
                    if body:
                        self._put(flat[:body], everyone, self.off + o, r, bases, tmo)
                else:  # large: slice j to receiver j only (the source's NVLink egress carries it once)
                    for (lo, hi), m in zip(parts, receivers):
                        if hi > lo:
                            self._put(flat[lo:hi], 1 << m, self.off + o + lo, r, bases, tmo)
                if nb - body:  # ragged tail: pad to one 16-byte vector
                    tail = torch.zeros(16, dtype=torch.uint8, device=flat.device)
                    tail[:nb - body] = flat[body:]
                    self._put(tail, everyone, self.off + o + body, r, bases, tmo)
        g.barrier(status)
        if g.rank != src_member and k >= 2:
            # all-gather among the receivers: each forwards its slice to the others
            j = receivers.index(g.rank)
            others = 0
            for m in receivers:
                if m != g.rank:
                    others |= 1 << m
            for o, nb in zip(offs, sizes):
                _, parts = split(nb)
                if parts is None:
                    continue
                lo, hi = parts[j]
                if hi > lo:
                    mine = self.heap.tensor[self.off + o + lo:self.off + o + hi]
                    self._put(mine, others, self.off + o + lo, r, bases, tmo)
        if k >= 2 and any(split(nb)[1] is not None for nb in sizes):
            g.barrier(status)
        if g.rank == src_member:
            out = tensors
        else:
            out = []
            for (shape, dt), o, nb in zip(specs, offs, sizes):
                out.append(self.heap.tensor[self.off + o:self.off + o + nb].view(dt).view(shape).clone())
        g.barrier(status)  # the staging area may be reused after every receiver copied out
        check_status(self.heap.device)
        return _rebuild(desc, out)
