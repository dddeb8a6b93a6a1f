"""Symmetric heap: one device buffer per rank, mapped into every peer.

Each rank cudaMalloc's ``nbytes`` (zeroed) through the extension, exports a
CUDA IPC handle, and all ranks exchange handles over torch.distributed; every
rank then opens every peer's heap, so kernels receive plain device pointers
into peer memory.  Allocation inside the heap is a deterministic bump
allocator: all ranks call ``alloc`` in the same order and therefore get the
same offsets, which is what lets a kernel address "the same buffer" on a peer
as ``base[peer] + offset``.  The first FLAG_BYTES hold the per-channel barrier
flags.  Group registration is host-only (a list of member bases), so forming
a new rank group costs microseconds, not a communicator initialisation.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ..ops._ext import ext, kernel

_DTYPE_SIZE = {torch.bfloat16: 2, torch.float16: 2, torch.float32: 4, torch.int32: 4, torch.uint8: 1}


class SymmetricHeap:
    def __init__(self, nbytes: int, device: torch.device, group=None):
        self.device = device
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.nbytes = int(nbytes)
        self.tensor, handle = ext().symm_alloc(self.nbytes, device.index)
        handles = [None] * self.size
        dist.all_gather_object(handles, handle, group=group)
        self.bases: list[int] = []
        self._opened: list[int] = []
        for i, h in enumerate(handles):
            if i == self.rank:
                self.bases.append(self.tensor.data_ptr())
            else:
                p = ext().symm_open(h, device.index)
                self._opened.append(p)
                self.bases.append(p)
        self.cursor = max(int(ext().FLAG_BYTES), 65536)
        self.epochs: dict[int, int] = {}
        dist.barrier(group=group)

    def alloc(self, nbytes: int, align: int = 1024) -> int:
        off = int(math.ceil(self.cursor / align) * align)
        if off + nbytes > self.nbytes:
            raise MemoryError(f"symmetric heap exhausted ({off + nbytes} > {self.nbytes} bytes)")
        self.cursor = off + nbytes
        return off

    def view(self, offset: int, shape, dtype=torch.bfloat16) -> torch.Tensor:
        n = math.prod(shape) * _DTYPE_SIZE[dtype]
        return self.tensor[offset:offset + n].view(dtype).view(*shape)

    def alloc_view(self, shape, dtype=torch.bfloat16):
        off = self.alloc(math.prod(shape) * _DTYPE_SIZE[dtype])
        return off, self.view(off, shape, dtype)

    def next_epoch(self, channel: int) -> int:
        self.epochs[channel] = self.epochs.get(channel, 0) + 1
        return self.epochs[channel]

    def close(self):
        for p in self._opened:
            ext().symm_close(p)
        self._opened.clear()


class PeerGroup:
    """An ordered subset of heap ranks with its own flag channel."""

    def __init__(self, heap: SymmetricHeap, members: tuple, channel: int, timeout_s: float = 10.0):
        if heap.rank not in members:
            raise ValueError("this rank is not a member of the group")
        if not 0 <= channel < int(ext().CHANNELS):
            raise ValueError("channel out of range")
        self.heap = heap
        self.members = tuple(members)
        self.rank = self.members.index(heap.rank)
        self.size = len(self.members)
        self.bases = [heap.bases[m] for m in self.members]
        self.channel = channel
        self.timeout_ns = int(timeout_s * 1e9)

    def args(self):
        return self.rank, self.bases, self.timeout_ns

    def barrier(self, status):
        kernel("group_barrier")(self.rank, self.bases, self.timeout_ns, self.channel,
                            self.heap.next_epoch(self.channel), status)
