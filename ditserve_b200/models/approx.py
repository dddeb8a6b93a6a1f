"""Approximate-mode extras (opt-in research paths; exact mode never uses them).

* ``CFGFolding`` — late-step classifier-free-guidance folding.  With v = cond + (g-1) d,
  d = cond - uncond, the guidance delta d changes slowly late in sampling; once the
  relative change of d between steps stays under ``threshold`` (curvature gate) after a
  warm-up fraction of the schedule, the unconditional branch is skipped for the next
  ``fold_span`` steps and the last d is reused.  Under CFG parallelism the unconditional
  rank group is idle while folded, so the planner may give it to other work ("fission").
* ``BlockResidualCache`` — DBCache-style reuse of the middle blocks' residual: always run
  the first ``front`` and last ``back`` blocks; if the front residual moved less than
  ``threshold`` (relative L1) since it was last computed, skip the middle blocks and add
  the cached middle residual, extrapolated to first order (Taylor) from its last two values.
  Works for the Wan block stack (``run_wan``) and the SD3.5 joint blocks
  (``SD35Transformer.forward_packed(..., cache=...)`` through ``run_blocks``; the cache is
  reset whenever the packed batch's composition changes).
* ``int8 ring codec`` — per-token, per-head symmetric INT8 with an fp32 scale for the K/V
  chunks exchanged between ring ranks (128 bf16 = 256 B -> 128 B + 4 B); the codec itself,
  its anchor-step schedule and both transports live in ``parallel.ring_codec``; these
  helpers are its torch statement.
Reference: workers/ditserve/models/wan/cfg_reuse.py:19-411, taylor_cache.py:27-179,
ring_quant.py:18-171, models/sd35_cache.py:8-286.
"""
from __future__ import annotations

import torch


class CFGFolding:
    def __init__(self, steps: int, warm_frac: float = 0.5, threshold: float = 0.05, fold_span: int = 2):
        self.steps = steps
        self.warm = int(steps * warm_frac)
        self.threshold = threshold
        self.fold_span = fold_span
        self.delta: torch.Tensor | None = None
        self.prev_delta: torch.Tensor | None = None
        self.folded_left = 0
        self.folded_steps = 0
        self.full_steps = 0

    def fold_now(self, step: int) -> bool:
        return self.folded_left > 0 and self.delta is not None and step >= self.warm

    def combine(self, step: int, guidance: float, cond: torch.Tensor, uncond: torch.Tensor | None) -> torch.Tensor:
        """Velocity for this step; ``uncond`` is None when the step was folded."""
        if uncond is None:
            if self.delta is None:
                raise RuntimeError("cannot fold before a full CFG step")
            self.folded_left -= 1
            self.folded_steps += 1
            return cond.float() + (guidance - 1.0) * self.delta
        d = cond.float() - uncond.float()
        self.observe(step, d)
        return uncond.float() + guidance * d

    def observe(self, step: int, d: torch.Tensor):
        """Record the guidance delta of a full CFG step (also fed by the fused CFG-parallel
        kernel, which writes cond - uncond while it applies the step) and run the gate."""
        self.prev_delta, self.delta = self.delta, d.float().clone()
        self.full_steps += 1
        if self.prev_delta is not None and step >= self.warm:
            change = ((self.delta - self.prev_delta).norm() / self.delta.norm().clamp_min(1e-12)).item()
            if change < self.threshold:
                self.folded_left = self.fold_span

    def eligible(self, step: int) -> bool:
        """The next step may run folded (the planner can hand the unconditional half away)."""
        return self.fold_now(step)


class BlockResidualCache:
    def __init__(self, layers: int, front: int = 2, back: int = 2, threshold: float = 0.08, max_reuse: int = 3):
        if front + back >= layers:
            raise ValueError("front + back must leave middle blocks to cache")
        self.layers, self.front, self.back = layers, front, back
        self.threshold = threshold
        self.max_reuse = max_reuse
        self.front_res: torch.Tensor | None = None
        self.mid_res: list = []
        self.reused = 0
        self.skipped_blocks = 0

    def middle(self) -> range:
        return range(self.front, self.layers - self.back)

    def should_skip(self, front_residual: torch.Tensor) -> bool:
        if self.front_res is None or len(self.mid_res) == 0 or self.reused >= self.max_reuse:
            return False
        rel = ((front_residual - self.front_res).abs().mean() / self.front_res.abs().mean().clamp_min(1e-12)).item()
        return rel < self.threshold

    def predicted_middle(self) -> torch.Tensor:
        if len(self.mid_res) >= 2:
            return 2 * self.mid_res[-1] - self.mid_res[-2]  # first-order Taylor step
        return self.mid_res[-1]

    def record(self, front_residual: torch.Tensor, mid_residual: torch.Tensor | None):
        self.front_res = front_residual.detach().clone()
        if mid_residual is not None:
            self.mid_res = (self.mid_res + [mid_residual.detach().clone()])[-2:]
            self.reused = 0
        else:
            self.reused += 1

    def run_blocks(self, block_fn, x: torch.Tensor, key=None) -> torch.Tensor:
        """Generic block stack: ``block_fn(i, x) -> x`` for i < layers, with middle reuse."""
        if key is not None and key != getattr(self, "_key", None):
            self.front_res, self.mid_res, self.reused, self._key = None, [], 0, key
        x_in = x.clone()  # block_fn may update x in place
        for i in range(self.front):
            x = block_fn(i, x)
        front_residual = x.float() - x_in.float()
        if self.should_skip(front_residual):
            x.copy_((x.float() + self.predicted_middle()).to(x.dtype))
            self.skipped_blocks += len(self.middle())
            self.record(front_residual, None)
        else:
            x_mid = x.clone()
            for i in self.middle():
                x = block_fn(i, x)
            self.record(front_residual, x.float() - x_mid.float())
        for i in range(self.layers - self.back, self.layers):
            x = block_fn(i, x)
        return x

    def run_wan(self, model, pk, pctx=None):
        """One Wan forward over the block stack with middle-block reuse (packet updated)."""
        x_in = pk.x.clone()
        for i in range(self.front):
            model.forward_block(i, pk, pctx)
        front_residual = (pk.x.float() - x_in.float())
        if self.should_skip(front_residual):
            pk.x = (pk.x.float() + self.predicted_middle()).to(pk.x.dtype)
            self.skipped_blocks += len(self.middle())
            self.record(front_residual, None)
        else:
            x_mid = pk.x.clone()
            for i in self.middle():
                model.forward_block(i, pk, pctx)
            self.record(front_residual, pk.x.float() - x_mid.float())
        for i in range(self.layers - self.back, self.layers):
            model.forward_block(i, pk, pctx)
        pk.next_block = self.layers
        return pk


def quantize_int8(x: torch.Tensor, head_dim: int):
    """Ring K/V codec, encode side (see ``parallel.ring_codec``)."""
    from ..parallel.ring_codec import RingInt8Codec
    return RingInt8Codec.encode(x, head_dim)


def dequantize_int8(q: torch.Tensor, scale: torch.Tensor, head_dim: int, dtype=torch.bfloat16):
    """Ring K/V codec, decode side (see ``parallel.ring_codec``)."""
    from ..parallel.ring_codec import RingInt8Codec
    return RingInt8Codec.decode(q, scale, head_dim, dtype)


def packet_bytes(tokens: int, heads: int, head_dim: int, int8: bool) -> int:
    """Bytes of ``tokens`` x ``heads`` vectors of one of K or V on the wire."""
    from ..parallel.ring_codec import RingInt8Codec
    return RingInt8Codec.wire_bytes(tokens, heads, head_dim, int8) // 2
