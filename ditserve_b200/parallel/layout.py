"""Parallel forms and rank layouts (CFG x Ulysses x ring) for one request group.

``Form(cfg, sp, ring)`` names follow the reference's planner vocabulary
(``sp4``, ``cfg2``, ``cfg2sp4``, ``u2r2``, ``cfg2u2r2``;
src/ditserve/control/cluster.cpp:78-109).  ``FixedLayout`` maps a group of
global ranks onto CFG roles and SP sub-groups: with cfg = 2 the first half of
the group computes the conditional branch and the second half the
unconditional one (reference: workers/ditserve/models/wan/parallel.py:123-170).
On NVSwitch every rank subset is equally connected, so groups need no
topology alignment; they are still kept contiguous for readability.
"""
from __future__ import annotations

import re
from dataclasses import dataclass

SP_DEGREES = (1, 2, 3, 4, 6, 8)


@dataclass(frozen=True)
class Form:
    cfg: int = 1
    sp: int = 1
    ring: int = 1

    @property
    def gpus(self) -> int:
        return self.cfg * self.sp

    @property
    def ulysses(self) -> int:
        return self.sp // self.ring

    @property
    def name(self) -> str:
        if self.ring > 1:
            base = f"u{self.ulysses}r{self.ring}"
        else:
            base = f"sp{self.sp}"
        if self.cfg == 2:
            return "cfg2" if self.sp == 1 else "cfg2" + base
        return base

    @classmethod
    def parse(cls, name: str) -> "Form":
        m = re.fullmatch(r"(cfg2)?(?:sp(\d+)|u(\d+)r(\d+))?", name)
        if not m or name == "":
            raise ValueError(f"bad form name {name!r}")
        cfg = 2 if m.group(1) else 1
        if m.group(2):
            sp, ring = int(m.group(2)), 1
        elif m.group(3):
            u, ring = int(m.group(3)), int(m.group(4))
            sp = u * ring
        else:
            sp, ring = 1, 1
        form = cls(cfg, sp, ring)
        form.validate()
        return form

    def validate(self, heads: int | None = None):
        if self.cfg not in (1, 2):
            raise ValueError("cfg degree must be 1 or 2")
        if self.sp < 1 or self.ring < 1 or self.sp % self.ring:
            raise ValueError("sp must be a multiple of ring")
        if self.ring > 1 and self.sp < 4:
            raise ValueError("ring attention needs sp >= 4")
        if heads is not None and heads % self.ulysses:
            raise ValueError(f"{heads} heads do not split over ulysses degree {self.ulysses}")
        return self


@dataclass(frozen=True)
class FixedLayout:
    ranks: tuple
    form: Form
    epoch: int = 0

    def __post_init__(self):
        if len(self.ranks) != self.form.gpus:
            raise ValueError("layout ranks must match the form's GPU count")

    def cfg_role(self, rank: int) -> int:
        return 0 if self.form.cfg == 1 else self.ranks.index(rank) // self.form.sp

    def sp_ranks(self, rank: int) -> tuple:
        i = self.ranks.index(rank) // self.form.sp
        return tuple(self.ranks[i * self.form.sp:(i + 1) * self.form.sp])

    def cfg_partner(self, rank: int) -> int | None:
        if self.form.cfg == 1:
            return None
        i = self.ranks.index(rank)
        return self.ranks[(i + self.form.sp) % len(self.ranks)]

    def sp_rank(self, rank: int) -> int:
        return self.sp_ranks(rank).index(rank)

    # Ulysses x ring inside one SP group: member m = r * U + u holds token shard m of the
    # sequence; the U-group (same r) exchanges heads, the ring group (same u) shares keys.
    def ulysses_ranks(self, rank: int) -> tuple:
        sp = self.sp_ranks(rank)
        U = self.form.ulysses
        r = sp.index(rank) // U
        return tuple(sp[r * U:(r + 1) * U])

    def ring_ranks(self, rank: int) -> tuple:
        sp = self.sp_ranks(rank)
        U = self.form.ulysses
        u = sp.index(rank) % U
        return tuple(sp[rr * U + u] for rr in range(self.form.ring))


def default_form(n_gpus: int, cfg: bool = True) -> Form:
    """Best single-request form on NVSwitch: CFG parallelism first, then Ulysses."""
    if cfg and n_gpus >= 2 and n_gpus % 2 == 0:
        return Form(2, n_gpus // 2, 1)
    return Form(1, n_gpus, 1)


def aligned_groups(world: int, size: int) -> list[tuple]:
    """Contiguous rank groups of ``size`` covering ``world`` (3/6-rank groups allowed)."""
    return [tuple(range(i, i + size)) for i in range(0, world - size + 1, size)]
