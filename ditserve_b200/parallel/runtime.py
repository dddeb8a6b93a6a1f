"""Process-group construction for a FixedLayout and selection of the collective path.

Every rank calls ``build_parallel`` with the same layout: it creates the SP
sub-groups and CFG pairs in one fixed order (``new_group`` is collective) and
returns ``(pctx, cfg_plan)`` for the Wan engine.  ``attention="nccl"`` is the
NCCL baseline; ``attention="fused"`` uses the peer-memory kernels of
``parallel.fused`` when they are available for the layout.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..models.wan.model import LocalAttention
from ..models.wan.runtime import CFGLocal
from .layout import FixedLayout
from .nccl import CFGExchangeNCCL, UlyssesNCCL, UlyssesRingNCCL


def build_parallel(layout: FixedLayout, rank: int, device: torch.device, attention: str = "fused",
                   seq_local: int | None = None, cfg=None, pred_numel: int | None = None):
    form = layout.form
    sp_groups, cfg_groups = {}, {}
    n_sp = len(layout.ranks) // form.sp
    for i in range(n_sp):
        ranks = layout.ranks[i * form.sp:(i + 1) * form.sp]
        g = dist.new_group(list(ranks)) if form.sp > 1 else None
        sp_groups[ranks] = g
    if form.cfg == 2:
        for j in range(form.sp):
            pair = (layout.ranks[j], layout.ranks[j + form.sp])
            cfg_groups[pair] = dist.new_group(list(pair))
    u_groups, ring_groups = {}, {}
    if form.ring > 1:
        U, R = form.ulysses, form.ring
        for i in range(n_sp):
            sp = layout.ranks[i * form.sp:(i + 1) * form.sp]
            for r in range(R):
                g = tuple(sp[r * U:(r + 1) * U])
                u_groups[g] = dist.new_group(list(g)) if U > 1 else None
            for u in range(U):
                g = tuple(sp[rr * U + u] for rr in range(R))
                ring_groups[g] = dist.new_group(list(g))
    pctx = LocalAttention()
    cfg_plan = CFGLocal()
    my_sp = layout.sp_ranks(rank)
    if form.sp > 1 and form.ring > 1:
        pctx = UlyssesRingNCCL(sp_groups[my_sp], u_groups[layout.ulysses_ranks(rank)],
                               ring_groups[layout.ring_ranks(rank)], form.sp, layout.sp_rank(rank), form.ulysses,
                               form.ring)
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
                                           seq_local=seq_local, cfg=cfg, pred_numel=pred_numel)
    return pctx, cfg_plan
