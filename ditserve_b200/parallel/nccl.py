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
