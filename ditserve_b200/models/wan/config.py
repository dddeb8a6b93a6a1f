"""Wan DiT configurations (shapes of the public diffusers checkpoints).

Wan2.1-T2V-1.3B and Wan2.2-TI2V-5B as served by the reference
(workers/ditserve/evaluation/cost_profile.py:16-23; results/5.1_Experimental_Setup/README.md:26-35),
plus the tiny 2-block model used for the CPU/Gloo contract gates.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass


@dataclass(frozen=True)
class WanConfig:
    name: str
    dim: int
    heads: int
    ffn_dim: int
    layers: int
    in_channels: int
    out_channels: int
    patch: tuple = (1, 2, 2)
    text_dim: int = 4096
    text_len: int = 512
    freq_dim: int = 256
    eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_max_seq: int = 1024
    flow_shift: float = 3.0
    expand_timesteps: bool = False   # Wan2.2 TI2V: per-token timesteps
    vae_stride: tuple = (4, 8, 8)

    @property
    def head_dim(self) -> int:
        return self.dim // self.heads

    def tokens(self, latent_shape) -> int:
        c, f, h, w = latent_shape
        return (f // self.patch[0]) * (h // self.patch[1]) * (w // self.patch[2])

    def to_dict(self) -> dict:
        return asdict(self)


WAN21_T2V_1_3B = WanConfig("wan2.1-t2v-1.3b", dim=1536, heads=12, ffn_dim=8960, layers=30,
                           in_channels=16, out_channels=16)
WAN22_TI2V_5B = WanConfig("wan2.2-ti2v-5b", dim=3072, heads=24, ffn_dim=14336, layers=30,
                          in_channels=48, out_channels=48, expand_timesteps=True, flow_shift=5.0,
                          vae_stride=(4, 16, 16))
WAN_TINY = WanConfig("wan-tiny", dim=128, heads=4, ffn_dim=512, layers=2, in_channels=16, out_channels=16,
                     text_dim=64, text_len=16)

CONFIGS = {c.name: c for c in (WAN21_T2V_1_3B, WAN22_TI2V_5B, WAN_TINY)}

# latent shapes (C, F, H, W) of the request tiers used in the studies
LATENTS = {
    ("wan2.1-t2v-1.3b", "480p"): (16, 21, 60, 104),     # 832x480, 81 frames -> 32 760 tokens
    ("wan2.1-t2v-1.3b", "720p"): (16, 21, 90, 160),     # 1280x720, 81 frames -> 75 600 tokens
    ("wan2.1-t2v-1.3b", "240p"): (16, 21, 30, 52),
    ("wan2.2-ti2v-5b", "720p"): (48, 31, 44, 80),       # 1280x704, 121 frames -> 27 280 tokens
    ("wan2.2-ti2v-5b", "480p"): (48, 31, 30, 56),       # 13 888 tokens... rounded tier
    ("wan-tiny", "tiny"): (16, 4, 8, 8),
}
