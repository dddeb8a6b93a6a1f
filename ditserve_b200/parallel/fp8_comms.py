"""FP8 (e4m3) payloads for the Ulysses all-to-alls of the NCCL path, with per-layer calibration.

Each all-to-all row of one head (``head_dim`` values of one token's q, k, v or attention
output) travels as ``head_dim`` e4m3 bytes plus its fp32 scale (absmax / 448, the largest
finite e4m3 value), so a bf16 payload of 2 * head_dim bytes shrinks to head_dim + 4 (0.52x
at head_dim 128).  The quantisation error is bounded per row by the e4m3 mantissa (3 bits:
relative error <= 2^-4 after rounding), which is why it is applied per layer: ``calibrate``
runs each block of a probe packet once with bf16 and once with FP8 payloads, from the same
input, and keeps FP8 only for the blocks whose output stays within ``max_rel_error``.

The fused peer-memory kernels move bf16 (NVLink 5 is rarely the bound at these sizes); this
plan serves links where bytes dominate (PCIe, multi-node).  Reference: the FP8 communication
calibration of the reference's parallel engine (workers/xfuser/core/distributed/fp8_comms.py:487-530).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from .nccl import UlyssesNCCL

E4M3_MAX = 448.0  # largest finite float8 e4m3 (OCP FP8 format)


def fp8_pack(x: torch.Tensor) -> torch.Tensor:
    """[rows, d] -> uint8 [rows, d + 4]: e4m3 payload then the fp32 row scale."""
    xf = x.float()
    scale = (xf.abs().amax(dim=1) / E4M3_MAX).clamp_min(1e-30)
    q = (xf / scale[:, None]).to(torch.float8_e4m3fn).view(torch.uint8)
    return torch.cat([q, scale.contiguous().view(torch.uint8).view(-1, 4)], dim=1)


def fp8_unpack(buf: torch.Tensor, d: int, dtype=torch.bfloat16) -> torch.Tensor:
    """uint8 [rows, d + 4] -> [rows, d] in ``dtype``."""
    q = buf[:, :d].contiguous().view(torch.float8_e4m3fn).float()
    scale = buf[:, d:].contiguous().view(torch.float32).view(-1)
    return (q * scale[:, None]).to(dtype)


def payload_bytes(rows: int, d: int, fp8: bool) -> int:
    return rows * (d + 4) if fp8 else rows * d * 2


class FP8UlyssesNCCL(UlyssesNCCL):
    """Ulysses all-to-alls with FP8 payloads on the blocks in ``layers`` (None: every block)."""

    def __init__(self, group, sp_size: int, sp_rank: int, layers=None):
        super().__init__(group, sp_size, sp_rank)
        self.layers = None if layers is None else set(layers)
        self.block = None
        self.bytes_sent = 0

    def begin_block(self, i: int) -> None:
        self.block = i

    def _fp8_now(self) -> bool:
        return self.layers is None or self.block in self.layers

    def _a2a(self, send: torch.Tensor, d: int) -> torch.Tensor:
        """all-to-all of ``send`` [P, ...] whose rows are heads of width d."""
        P = self.sp_size
        if not self._fp8_now():
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=self.group)
            self.bytes_sent += send.numel() * send.element_size()
            return recv
        rows = send.numel() // d
        packed = fp8_pack(send.reshape(rows, d)).view(P, rows // P, d + 4)
        got = torch.empty_like(packed)
        dist.all_to_all_single(got, packed, group=self.group)
        self.bytes_sent += packed.numel()
        return fp8_unpack(got.view(rows, d + 4), d, send.dtype).view(send.shape)

    def self_attention_qkv(self, qkv: torch.Tensor, heads: int, batch: int, seq_local: int) -> torch.Tensor:
        P = self.sp_size
        hd = qkv.shape[1] // (3 * heads)
        hl = heads // P
        send = qkv.view(batch, seq_local, 3, P, hl, hd).permute(3, 0, 1, 2, 4, 5).contiguous()
        recv = self._a2a(send, hd)
        full = recv.permute(1, 0, 2, 3, 4, 5).reshape(batch, P * seq_local, 3, hl * hd)
        o = ops.attention(full[:, :, 0], full[:, :, 1], full[:, :, 2], hl)
        send2 = o.view(batch, P, seq_local, hl * hd).permute(1, 0, 2, 3).contiguous()
        recv2 = self._a2a(send2, hd)
        return recv2.permute(1, 2, 0, 3).reshape(batch * seq_local, heads * hd)


@torch.no_grad()
def calibrate(model, packet, plan: FP8UlyssesNCCL, max_rel_error: float = 0.02) -> dict:
    """Per-block choice between bf16 and FP8 payloads on one probe packet.

    Every rank of the SP group runs this with its shard of the same packet; the decision per
    block is the group's maximum error, so all ranks enable the same blocks.  Returns
    {"layers": [...], "errors": {block: rel_L2}}; ``plan.layers`` is set to the chosen blocks."""
    import dataclasses
    errors = {}
    pk = packet
    for i in range(len(model.blocks)):
        plan.layers = set()
        plan.begin_block(i)
        ref = model.forward_block(i, dataclasses.replace(pk, x=pk.x.clone()), plan)
        plan.layers = None
        plan.begin_block(i)
        got = model.forward_block(i, dataclasses.replace(pk, x=pk.x.clone()), plan)
        num = (got.x.float() - ref.x.float()).pow(2).sum()
        den = ref.x.float().pow(2).sum()
        both = torch.stack([num, den]).to(torch.float64)
        if plan.group is not None:
            dist.all_reduce(both, group=plan.group)
        err = float((both[0] / both[1].clamp_min(1e-30)).sqrt())
        errors[i] = err
        pk = ref  # the next block sees the exact input
    chosen = sorted(i for i, e in errors.items() if e <= max_rel_error)
    plan.layers = set(chosen)
    return dict(layers=chosen, errors=errors)
