"""NCCL reference path for the sequence/CFG collectives (the baseline the
fused peer-memory kernels are measured against).

* ``UlyssesNCCL`` — head<->sequence all-to-all around attention
  (reference: workers/xfuser/model_executor/layers/usp.py:207-270, :368-381).
* ``CFGExchangeNCCL`` — all-gather of the branch predictions inside a CFG pair
  (reference: workers/ditserve/models/xdit/wan.py:187-203).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops


class UlyssesNCCL:
    def __init__(self, group, sp_size: int, sp_rank: int):
        self.group = group
        self.sp_size = sp_size
        self.sp_rank = sp_rank

    def self_attention_qkv(self, qkv: torch.Tensor, heads: int, batch: int, seq_local: int) -> torch.Tensor:
        P = self.sp_size
        width3 = qkv.shape[1]
        hd = width3 // (3 * heads)
        hl = heads // P
        # [B, Sl, 3, P, hl, d] -> [P, B, Sl, 3, hl, d]: chunk j holds rank j's heads
        send = qkv.view(batch, seq_local, 3, P, hl, hd).permute(3, 0, 1, 2, 4, 5).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        # recv[src] = src's tokens for my heads -> [B, S, 3, hl*d]
        full = recv.permute(1, 0, 2, 3, 4, 5).reshape(batch, P * seq_local, 3, hl * hd)
        q, k, v = full[:, :, 0], full[:, :, 1], full[:, :, 2]
        o = ops.attention(q, k, v, hl)  # [B, S, hl*d]
        send2 = o.view(batch, P, seq_local, hl * hd).permute(1, 0, 2, 3).contiguous()
        recv2 = torch.empty_like(send2)
        dist.all_to_all_single(recv2, send2, group=self.group)
        return recv2.permute(1, 2, 0, 3).reshape(batch * seq_local, heads * hd)

    def self_attention(self, q, k, v, heads, batch, seq_local):
        qkv = torch.cat([q, k, v], dim=1)
        return self.self_attention_qkv(qkv, heads, batch, seq_local)

    def gather_sequence(self, y: torch.Tensor, batch: int, seq_local: int) -> torch.Tensor:
        P = self.sp_size
        parts = torch.empty((P * batch * seq_local, y.shape[1]), device=y.device, dtype=y.dtype)
        dist.all_gather_into_tensor(parts, y.contiguous(), group=self.group)
        return parts.view(P, batch, seq_local, -1).permute(1, 0, 2, 3).reshape(batch * P * seq_local, -1)


class CFGExchangeNCCL:
    def __init__(self, group, cfg_rank: int):
        self.group = group
        self.cfg_size = 2
        self.cfg_rank = cfg_rank

    def exchange(self, mine: torch.Tensor) -> torch.Tensor:
        flat = mine.contiguous().reshape(1, -1)
        both = torch.empty((2, flat.shape[1]), device=mine.device, dtype=mine.dtype)
        dist.all_gather_into_tensor(both, flat, group=self.group)
        return both[1 - self.cfg_rank].view(mine.shape)


class UlyssesRingNCCL(UlyssesNCCL):
    """NCCL baseline of Ulysses x ring: all-to-all inside the U-group, then the ring
    group's key/value chunks gathered and attended to in one pass (the exact result of a
    ring rotation with log-sum-exp merging).  With an INT8 ring codec active for the step,
    the chunks travel as int8 values plus fp32 scales (``parallel.ring_codec``)."""

    def __init__(self, sp_group, u_group, ring_group, sp_size, sp_rank, ulysses, ring, codec=None):
        self.group = u_group
        self.u_size = ulysses
        self.sp_group = sp_group
        self.ring_group = ring_group
        self.ring = ring
        self.sp_size = sp_size          # the model shards the sequence over the whole SP group
        self.sp_rank = sp_rank
        self.sp_size_total = sp_size
        self.ring_rank = sp_rank // ulysses
        self.codec = codec              # parallel.ring_codec.RingInt8Codec or None

    def set_step(self, step: int, total_steps: int):
        if self.codec is not None:
            self.codec.set_step(step, total_steps)

    def _gather_ring_kv(self, kv: torch.Tensor, hd: int) -> torch.Tensor:
        """All ring members' [B, chunk, 2, w] key/value chunks, stacked on a new leading axis."""
        parts = torch.empty((self.ring, *kv.shape), device=kv.device, dtype=kv.dtype)
        if self.codec is None or not self.codec.active:
            dist.all_gather_into_tensor(parts.view(self.ring * kv.shape[0], *kv.shape[1:]), kv, group=self.ring_group)
            if self.codec is not None:
                self.codec.account(kv.shape[0] * kv.shape[1], kv.shape[-1] // hd, hd, False, self.ring - 1)
            return parts
        q8, sc = self.codec.encode(kv, hd)
        q_all = torch.empty((self.ring, *q8.shape), device=kv.device, dtype=q8.dtype)
        s_all = torch.empty((self.ring, *sc.shape), device=kv.device, dtype=sc.dtype)
        dist.all_gather_into_tensor(q_all.view(self.ring * q8.shape[0], *q8.shape[1:]), q8, group=self.ring_group)
        dist.all_gather_into_tensor(s_all.view(self.ring * sc.shape[0], *sc.shape[1:]), sc, group=self.ring_group)
        parts.copy_(self.codec.decode(q_all, s_all, hd, kv.dtype))
        parts[self.ring_rank] = kv  # the local chunk stays exact
        self.codec.account(kv.shape[0] * kv.shape[1], kv.shape[-1] // hd, hd, True, self.ring - 1)
        return parts

    def self_attention_qkv(self, qkv, heads, batch, seq_local):
        U = self.u_size
        hd = qkv.shape[1] // (3 * heads)
        hl = heads // U
        if U > 1:
            send = qkv.view(batch, seq_local, 3, U, hl, hd).permute(3, 0, 1, 2, 4, 5).contiguous()
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=self.group)
            chunk = recv.permute(1, 0, 2, 3, 4, 5).reshape(batch, U * seq_local, 3, hl * hd)
        else:
            chunk = qkv.view(batch, seq_local, 3, heads * hd)
        kv = chunk[:, :, 1:].contiguous()
        parts = self._gather_ring_kv(kv, hd)
        keys = parts.permute(1, 0, 2, 3, 4).reshape(batch, self.ring * U * seq_local, 2, hl * hd)
        o = ops.attention(chunk[:, :, 0], keys[:, :, 0], keys[:, :, 1], hl)
        if U == 1:
            return o.reshape(batch * seq_local, heads * hd)
        send2 = o.view(batch, U, seq_local, hl * hd).permute(1, 0, 2, 3).contiguous()
        recv2 = torch.empty_like(send2)
        dist.all_to_all_single(recv2, send2, group=self.group)
        return recv2.permute(1, 2, 0, 3).reshape(batch * seq_local, heads * hd)

    def gather_sequence(self, y, batch, seq_local):
        P = self.sp_size_total
        parts = torch.empty((P * batch * seq_local, y.shape[1]), device=y.device, dtype=y.dtype)
        dist.all_gather_into_tensor(parts, y.contiguous(), group=self.sp_group)
        return parts.view(P, batch, seq_local, -1).permute(1, 0, 2, 3).reshape(batch * P * seq_local, -1)
