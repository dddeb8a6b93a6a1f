"""SD3.5 2-D VAE decoder (16 latent channels, 8x spatial upsampling).

Layout and parameter names follow diffusers ``AutoencoderKL`` as configured for SD3/SD3.5
(``decoder.conv_in``, ``decoder.mid_block.{resnets.0,attentions.0,resnets.1}``,
``decoder.up_blocks.i.{resnets.j,upsamplers.0.conv}``, ``decoder.conv_norm_out``,
``decoder.conv_out``; block channels 128/256/512/512, three resnets per up block, GroupNorm
with 32 groups, SiLU; no post-quant conv), so the checkpoint's ``vae/`` weights load with
``load_state_dict``.  Latents are un-scaled as ``z / scaling_factor + shift_factor``
(1.5305 and 0.0609 for SD3.5) before decoding.

The convolutions are cuDNN (library) calls; the mid-block attention over the latent-resolution
feature map (one 512-wide head) runs through torch SDPA.  Reference: the rank-0 image decode
of the SD3.5 worker (workers/ditserve/models/sd35.py, ``vae.decode`` after the denoise loop).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

SD35_SCALING = 1.5305
SD35_SHIFT = 0.0609


class ResnetBlock(nn.Module):
    def __init__(self, cin: int, cout: int, groups: int = 32, eps: float = 1e-6):
        super().__init__()
        self.norm1 = nn.GroupNorm(groups, cin, eps=eps)
        self.conv1 = nn.Conv2d(cin, cout, 3, padding=1)
        self.norm2 = nn.GroupNorm(groups, cout, eps=eps)
        self.conv2 = nn.Conv2d(cout, cout, 3, padding=1)
        self.conv_shortcut = nn.Conv2d(cin, cout, 1) if cin != cout else None

    def forward(self, x):
        h = self.conv1(F.silu(self.norm1(x)))
        h = self.conv2(F.silu(self.norm2(h)))
        if self.conv_shortcut is not None:
            x = self.conv_shortcut(x)
        return x + h


class AttnBlock(nn.Module):
    """Single-head spatial self-attention with a residual (diffusers ``Attention`` names)."""

    def __init__(self, dim: int, groups: int = 32, eps: float = 1e-6):
        super().__init__()
        self.group_norm = nn.GroupNorm(groups, dim, eps=eps)
        self.to_q = nn.Linear(dim, dim)
        self.to_k = nn.Linear(dim, dim)
        self.to_v = nn.Linear(dim, dim)
        self.to_out = nn.ModuleList([nn.Linear(dim, dim)])

    def forward(self, x):
        b, c, h, w = x.shape
        t = self.group_norm(x).flatten(2).transpose(1, 2)  # [B, HW, C]
        q, k, v = self.to_q(t), self.to_k(t), self.to_v(t)
        o = F.scaled_dot_product_attention(q[:, None], k[:, None], v[:, None])[:, 0]
        o = self.to_out[0](o)
        return x + o.transpose(1, 2).reshape(b, c, h, w)


class MidBlock(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.resnets = nn.ModuleList([ResnetBlock(dim, dim), ResnetBlock(dim, dim)])
        self.attentions = nn.ModuleList([AttnBlock(dim)])

    def forward(self, x):
        x = self.resnets[0](x)
        x = self.attentions[0](x)
        return self.resnets[1](x)


class Upsample(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.conv = nn.Conv2d(dim, dim, 3, padding=1)

    def forward(self, x):
        return self.conv(F.interpolate(x, scale_factor=2.0, mode="nearest"))


class UpBlock(nn.Module):
    def __init__(self, cin: int, cout: int, layers: int, upsample: bool):
        super().__init__()
        self.resnets = nn.ModuleList([ResnetBlock(cin if i == 0 else cout, cout) for i in range(layers)])
        self.upsamplers = nn.ModuleList([Upsample(cout)]) if upsample else None

    def forward(self, x):
        for r in self.resnets:
            x = r(x)
        if self.upsamplers is not None:
            x = self.upsamplers[0](x)
        return x


class Decoder(nn.Module):
    def __init__(self, z: int = 16, out: int = 3, channels=(128, 256, 512, 512), layers: int = 2):
        super().__init__()
        rev = list(reversed(channels))
        self.conv_in = nn.Conv2d(z, rev[0], 3, padding=1)
        self.mid_block = MidBlock(rev[0])
        blocks = []
        prev = rev[0]
        for i, ch in enumerate(rev):
            blocks.append(UpBlock(prev, ch, layers + 1, upsample=i < len(rev) - 1))
            prev = ch
        self.up_blocks = nn.ModuleList(blocks)
        self.conv_norm_out = nn.GroupNorm(32, channels[0], eps=1e-6)
        self.conv_out = nn.Conv2d(channels[0], out, 3, padding=1)

    def forward(self, z):
        x = self.mid_block(self.conv_in(z))
        for blk in self.up_blocks:
            x = blk(x)
        return self.conv_out(F.silu(self.conv_norm_out(x)))


class SD35VAEDecoder(nn.Module):
    def __init__(self, z: int = 16, channels=(128, 256, 512, 512), scaling: float = SD35_SCALING,
                 shift: float = SD35_SHIFT):
        super().__init__()
        self.decoder = Decoder(z, 3, channels)
        self.scaling, self.shift = scaling, shift

    @classmethod
    def random_init(cls, device="cpu", dtype=torch.bfloat16, seed: int = 0, channels=(128, 256, 512, 512)):
        g = torch.Generator().manual_seed(seed)
        m = cls(channels=channels)
        with torch.no_grad():
            for name, p in m.named_parameters():
                if p.dim() > 1:
                    fan_in = p[0].numel()
                    p.copy_(torch.randn(p.shape, generator=g) / math.sqrt(fan_in))
                elif name.endswith("weight"):
                    p.fill_(1.0)
                else:
                    p.zero_()
        return m.to(device=device, dtype=dtype).eval()

    @torch.inference_mode()
    def decode(self, latents: torch.Tensor) -> torch.Tensor:
        """[B, 16, h, w] model-space latents -> [B, 3, 8h, 8w] images in [-1, 1] (clamped)."""
        z = latents.to(next(self.parameters()).dtype) / self.scaling + self.shift
        return self.decoder(z).clamp(-1, 1)
