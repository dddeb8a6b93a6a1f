"""Process-group construction for a FixedLayout and selection of the collective path.

The ranks of a layout call ``build_parallel`` with the same layout; only they take part
(groups are created member-locally and cached by rank set, so other ranks of the world
can be busy with other requests meanwhile).  Returns ``(pctx, cfg_plan)`` for the Wan
engine.  ``attention="nccl"`` is the NCCL baseline; ``attention="nccl-fp8"`` is the same
path with FP8 payloads on the Ulysses all-to-alls (``parallel.fp8_comms``; plain Ulysses
forms, ``fp8_layers`` picks the blocks, None = all); ``attention="fused"`` uses the
peer-memory kernels of ``parallel.fused`` when they are available for the layout.
``ring_codec`` ("int8" or a dict of ``RingInt8Codec`` options) sends the ring key/value
chunks of ring forms as int8 packets outside the bf16 anchor steps, on either path.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..models.wan.model import LocalAttention
from ..models.wan.runtime import CFGLocal
from .layout import FixedLayout
from .nccl import CFGExchangeNCCL, UlyssesNCCL, UlyssesRingNCCL


_GROUPS: dict = {}


def group_for(ranks):
    """Process group over ``ranks`` (None = the default group when it spans the world).

    Created member-locally (``use_local_synchronization``): only the member ranks call it,
    each rank set once per process (torch names such groups by a hash of the ranks).
    """
    key = tuple(sorted(int(r) for r in ranks))
    if len(key) == dist.get_world_size() and key == tuple(range(len(key))):
        return None
    if key not in _GROUPS:
        _GROUPS[key] = dist.new_group(list(key), use_local_synchronization=True)
    return _GROUPS[key]


def build_parallel(layout: FixedLayout, rank: int, device: torch.device, attention: str = "fused",
                   seq_local: int | None = None, cfg=None, pred_numel: int | None = None, fp8_layers=None,
                   ring_codec=None):
    if attention not in ("fused", "nccl", "nccl-fp8"):
        raise ValueError(f"unknown collective path {attention!r}")
    form = layout.form
    sp_groups, cfg_groups = {}, {}
    my_sp = layout.sp_ranks(rank)
    if form.sp > 1:
        sp_groups[my_sp] = group_for(my_sp)
    else:
        sp_groups[my_sp] = None
    if form.cfg == 2:
        pair = tuple(sorted((rank, layout.cfg_partner(rank))))
        cfg_groups[pair] = group_for(pair)
    u_groups, ring_groups = {}, {}
    if form.ring > 1:
        ug, rg = layout.ulysses_ranks(rank), layout.ring_ranks(rank)
        u_groups[ug] = group_for(ug) if len(ug) > 1 else None
        ring_groups[rg] = group_for(rg)
    pctx = LocalAttention()
    cfg_plan = CFGLocal()
    codec = None
    if form.ring > 1 and ring_codec is not None:
        from .ring_codec import make_codec
        codec = make_codec(ring_codec)
    if form.sp > 1 and form.ring > 1:
        pctx = UlyssesRingNCCL(sp_groups[my_sp], u_groups[layout.ulysses_ranks(rank)],
                               ring_groups[layout.ring_ranks(rank)], form.sp, layout.sp_rank(rank), form.ulysses,
                               form.ring, codec=codec)
    elif form.sp > 1 and attention == "nccl-fp8":
        from .fp8_comms import FP8UlyssesNCCL
        pctx = FP8UlyssesNCCL(sp_groups[my_sp], form.sp, layout.sp_rank(rank), layers=fp8_layers)
    elif form.sp > 1:
        pctx = UlyssesNCCL(sp_groups[my_sp], form.sp, layout.sp_rank(rank))
    if form.cfg == 2:
        partner = layout.cfg_partner(rank)
        pair = tuple(sorted((rank, partner)))
        cfg_plan = CFGExchangeNCCL(cfg_groups[pair], layout.cfg_role(rank))
    if attention == "fused":
        try:
            from . import fused
        except ImportError:
            fused = None
        if fused is not None:
            pctx, cfg_plan = fused.upgrade(layout, rank, device, pctx, cfg_plan, sp_groups, cfg_groups,
                                           seq_local=seq_local, cfg=cfg, pred_numel=pred_numel, codec=codec)
    return pctx, cfg_plan
