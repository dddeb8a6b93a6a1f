"""INT8 transport codec for the ring-attention key/value chunks, with bf16 anchor steps.

Under Ulysses x ring (2D USP) every ring rank needs the key/value chunks of its ring peers.
With the codec active, a chunk crosses the link as int8 values with one fp32 scale per
(token, head) vector: symmetric quantisation, scale = max|x| / 127 (floored at 1e-30),
q = clamp(round_half_even(x / scale), -127, 127), x' = q * scale rounded to bf16.  A vector
of 128 bf16 values (256 B) travels as 132 B.  The rank's own chunk stays exact.

Step-aware anchors keep the first ``warmup_steps`` and the last ``tail_anchor_steps``
denoising steps in bf16, where the trajectory is most sensitive (the reference's schedule:
workers/ditserve/models/wan/ring_quant.py:18-55).  Its bounded-drift gate (cos >= 0.95,
relL2 <= 0.25 against the bf16 ring) is what ``tests/test_ring_codec.py`` checks.

Two transports use the same arithmetic:
  * the NCCL baseline (``UlyssesRingNCCL``) all-gathers int8 values and fp32 scales and
    decodes them with ``decode`` (host-side torch ops);
  * the fused path (``FusedUSP``) quantizes once in ``ring_quant_push`` (a kernel that stores
    the packet into every ring peer's heap slot over NVLink) and decodes each slot locally with
    ``ring_dequant``; the attention kernel then reads the decoded chunks from local memory.
"""
from __future__ import annotations

import torch

SCALE_FLOOR = 1e-30


class RingInt8Codec:
    def __init__(self, warmup_steps: int = 2, tail_anchor_steps: int = 2, enabled: bool = True):
        self.warmup_steps = max(0, int(warmup_steps))
        self.tail_anchor_steps = max(0, int(tail_anchor_steps))
        self.enabled = bool(enabled)
        self.active = self.enabled
        self.stats = {"int8_chunks": 0, "bf16_chunks": 0, "orig_bytes": 0, "wire_bytes": 0}

    def should_quantize(self, step: int, total_steps: int) -> bool:
        if not self.enabled:
            return False
        return self.warmup_steps <= step < max(0, total_steps - self.tail_anchor_steps)

    def set_step(self, step: int, total_steps: int) -> bool:
        self.active = self.should_quantize(step, total_steps)
        return self.active

    @staticmethod
    def wire_bytes(rows: int, heads: int, head_dim: int, int8: bool) -> int:
        """Bytes of one K+V chunk of ``rows`` tokens on the wire."""
        per = heads * (head_dim + 4) if int8 else heads * head_dim * 2
        return 2 * rows * per

    def account(self, rows: int, heads: int, head_dim: int, int8: bool, chunks: int = 1):
        self.stats["int8_chunks" if int8 else "bf16_chunks"] += chunks
        self.stats["orig_bytes"] += chunks * self.wire_bytes(rows, heads, head_dim, False)
        self.stats["wire_bytes"] += chunks * self.wire_bytes(rows, heads, head_dim, int8)

    def summary(self) -> dict:
        orig, wire = max(1, self.stats["orig_bytes"]), max(1, self.stats["wire_bytes"])
        return {**self.stats, "compression_ratio": round(orig / wire, 4)}

    # -------------------------------------------------------------- torch statement
    @staticmethod
    def encode(x: torch.Tensor, head_dim: int) -> tuple[torch.Tensor, torch.Tensor]:
        """[..., H*D] -> (int8 [..., H*D], fp32 scales [..., H]) per token and head."""
        shp = x.shape
        h = shp[-1] // head_dim
        xf = x.float().reshape(*shp[:-1], h, head_dim)
        scale = xf.abs().amax(-1).clamp_min(SCALE_FLOOR) / 127.0
        q = torch.round(xf / scale[..., None]).clamp(-127, 127).to(torch.int8)
        return q.reshape(shp), scale

    @staticmethod
    def decode(q: torch.Tensor, scale: torch.Tensor, head_dim: int, dtype=torch.bfloat16) -> torch.Tensor:
        shp = q.shape
        h = shp[-1] // head_dim
        x = q.float().reshape(*shp[:-1], h, head_dim) * scale.float()[..., None]
        return x.reshape(shp).to(dtype)


def make_codec(spec) -> RingInt8Codec | None:
    """``None``/``"off"`` -> no codec; ``"int8"`` -> default anchors; a dict -> keyword options."""
    if spec in (None, False, "off", "none", "bf16"):
        return None
    if spec in (True, "int8"):
        return RingInt8Codec()
    if isinstance(spec, dict):
        opts = dict(spec)
        kind = opts.pop("kind", "int8")
        if kind != "int8":
            raise ValueError(f"unknown ring codec {kind!r}")
        return RingInt8Codec(**opts)
    raise ValueError(f"unknown ring codec {spec!r}")
