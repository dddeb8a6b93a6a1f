"""Wan causal 3-D VAE decoders: Wan2.1 (base 96, z 16, mults 1/2/4/4, 2 res blocks, 8x
spatial) and Wan2.2-TI2V (residual up blocks with duplicate-upsampling shortcuts, decoder
base 256, z 48, 12 output channels un-patchified 2x2 into RGB: 16x spatial).

Parameter names follow diffusers ``AutoencoderKLWan`` (``post_quant_conv``, ``decoder.conv_in``,
``decoder.mid_block.{resnets,attentions}``, ``decoder.up_blocks.i.{resnets,upsamplers}``,
``decoder.norm_out``, ``decoder.conv_out``) so its checkpoint loads with ``load_state_dict``.

Decoding is causal in time and runs one latent frame at a time: every causal conv keeps
the last two frames of its input in a feature cache, so ``ChunkedDecode`` can stop after
any latent frame and resume later with an identical result (the reference's chunked
decode, workers/ditserve/models/pipeline.py:171-231).  Frame 0 decodes to 1 video frame,
every later latent frame to 4 (two temporal x2 upsamplings).

Patch parallelism (``PatchParallel``): the frame is split over ranks along one spatial
axis; every 3x3 convolution first completes its input with one halo row/column from each
neighbour (peer-memory stores through ``halo_exchange`` or NCCL send/recv as baseline);
the mid-block attention all-gathers the (small) latent-resolution feature map.
"""
from __future__ import annotations


import torch
import torch.nn.functional as F
from torch import nn

CACHE_T = 2

WAN21_LATENTS_MEAN = [-0.7571, -0.7089, -0.9113, 0.1075, -0.1745, 0.9653, -0.1517, 1.5508,
                      0.4134, -0.0715, 0.5517, -0.3632, -0.1922, -0.9497, 0.2503, -0.2921]
WAN21_LATENTS_STD = [2.8184, 1.4541, 2.3275, 2.6558, 1.2196, 1.7708, 2.6052, 2.0743,
                     3.2687, 2.1526, 2.8652, 1.5579, 1.6382, 1.1253, 2.8251, 1.9160]


class Halo:
    """Spatial split of the decoder's feature maps across ranks (single rank: no-op)."""

    size = 1
    rank = 0
    axis = 3  # 3 = H, 4 = W of [B, C, T, H, W]

    def pad(self, x: torch.Tensor) -> torch.Tensor:
        """x with one halo slice on each side of the split axis (zeros at the frame edge)."""
        return x

    def gather(self, x: torch.Tensor) -> torch.Tensor:
        return x

    def local(self, x: torch.Tensor) -> torch.Tensor:
        return x


class CausalConv3d(nn.Conv3d):
    """Conv3d padded causally in time (2*p before, 0 after) and symmetrically in space."""

    def __init__(self, cin, cout, kernel, padding=0):
        super().__init__(cin, cout, kernel, padding=0)
        k = self.kernel_size
        p = padding if isinstance(padding, tuple) else (padding, padding, padding)
        self.tpad, self.hpad, self.wpad = 2 * p[0], p[1], p[2]

    def forward(self, x, cache=None, halo: Halo | None = None):
        tp = self.tpad
        if cache is not None and tp > 0:
            x = torch.cat([cache.to(x.dtype), x], dim=2)
            tp -= cache.shape[2]
        pad_h, pad_w = self.hpad, self.wpad
        if halo is not None and halo.size > 1 and (pad_h if halo.axis == 3 else pad_w) > 0:
            x = halo.pad(x)
            if halo.axis == 3:
                pad_h = 0
            else:
                pad_w = 0
        x = F.pad(x, (pad_w, pad_w, pad_h, pad_h, tp, 0))
        return F.conv3d(x, self.weight, self.bias)


class RMSNormC(nn.Module):
    """L2-normalise over channels, times sqrt(C) * gamma (+ bias)."""

    def __init__(self, dim, images=True, bias=False):
        super().__init__()
        shape = (dim, 1, 1) if images else (dim, 1, 1, 1)
        self.scale = dim ** 0.5
        self.gamma = nn.Parameter(torch.ones(shape))
        self.bias = nn.Parameter(torch.zeros(shape)) if bias else None

    def forward(self, x):
        y = F.normalize(x, dim=1) * self.scale * self.gamma
        return y + self.bias if self.bias is not None else y


class ResidualBlock(nn.Module):
    def __init__(self, cin, cout):
        super().__init__()
        self.norm1 = RMSNormC(cin, images=False)
        self.conv1 = CausalConv3d(cin, cout, 3, padding=1)
        self.norm2 = RMSNormC(cout, images=False)
        self.conv2 = CausalConv3d(cout, cout, 3, padding=1)
        self.conv_shortcut = CausalConv3d(cin, cout, 1) if cin != cout else None

    def _conv(self, conv, x, cache, idx, halo):
        new = x[:, :, -CACHE_T:].clone()
        old = cache[idx[0]]
        if new.shape[2] < 2 and old is not None:
            new = torch.cat([old[:, :, -1:].to(new.device), new], dim=2)
        out = conv(x, old, halo)
        cache[idx[0]] = new
        idx[0] += 1
        return out

    def forward(self, x, cache, idx, halo):
        h = self.conv_shortcut(x) if self.conv_shortcut is not None else x
        x = F.silu(self.norm1(x))
        x = self._conv(self.conv1, x, cache, idx, halo)
        x = F.silu(self.norm2(x))
        x = self._conv(self.conv2, x, cache, idx, halo)
        return x + h


class AttentionBlock(nn.Module):
    """Single-head spatial self-attention per frame (gathered across ranks)."""

    def __init__(self, dim):
        super().__init__()
        self.norm = RMSNormC(dim)
        self.to_qkv = nn.Conv2d(dim, dim * 3, 1)
        self.proj = nn.Conv2d(dim, dim, 1)

    def forward(self, x, halo):
        identity = x
        full = halo.gather(x)
        b, c, t, h, w = full.shape
        y = full.permute(0, 2, 1, 3, 4).reshape(b * t, c, h, w)
        y = self.norm(y)
        qkv = self.to_qkv(y).reshape(b * t, 3, c, h * w).permute(1, 0, 3, 2)  # [3, bt, hw, c]
        q, k, v = qkv[0], qkv[1], qkv[2]
        o = F.scaled_dot_product_attention(q.unsqueeze(1), k.unsqueeze(1), v.unsqueeze(1)).squeeze(1)
        o = o.permute(0, 2, 1).reshape(b * t, c, h, w)
        o = self.proj(o).view(b, t, c, h, w).permute(0, 2, 1, 3, 4)
        return halo.local(o) + identity


class Resample(nn.Module):
    """Nearest x2 spatial upsampling + 3x3 conv (to dim/2, or ``out_dim``); ``upsample3d``
    also doubles time."""

    def __init__(self, dim, mode, out_dim=None):
        super().__init__()
        self.mode = mode
        self.resample = nn.Sequential(nn.Upsample(scale_factor=(2.0, 2.0), mode="nearest-exact"),
                                      nn.Conv2d(dim, out_dim or dim // 2, 3, padding=1))
        if mode == "upsample3d":
            self.time_conv = CausalConv3d(dim, dim * 2, (3, 1, 1), padding=(1, 0, 0))

    def forward(self, x, cache, idx, halo):
        b, c, t, h, w = x.shape
        if self.mode == "upsample3d":
            i = idx[0]
            if cache[i] is None:
                cache[i] = "first"  # the first latent frame is not doubled in time
                idx[0] += 1
            else:
                new = x[:, :, -CACHE_T:].clone()
                if new.shape[2] < 2 and isinstance(cache[i], torch.Tensor):
                    new = torch.cat([cache[i][:, :, -1:].to(new.device), new], dim=2)
                if new.shape[2] < 2 and isinstance(cache[i], str):
                    new = torch.cat([torch.zeros_like(new), new], dim=2)
                x = self.time_conv(x) if isinstance(cache[i], str) else self.time_conv(x, cache[i])
                cache[i] = new
                idx[0] += 1
                x = x.reshape(b, 2, c, t, h, w)
                x = torch.stack((x[:, 0], x[:, 1]), 3).reshape(b, c, t * 2, h, w)
        t = x.shape[2]
        y = x.permute(0, 2, 1, 3, 4).reshape(b * t, c, h, w)
        y = F.interpolate(y.float(), scale_factor=2.0, mode="nearest-exact").to(x.dtype)
        conv = self.resample[1]
        if halo.size > 1:
            y5 = halo.pad(y.view(b, t, c, *y.shape[-2:]).permute(0, 2, 1, 3, 4))
            y = y5.permute(0, 2, 1, 3, 4).reshape(b * t, c, *y5.shape[-2:])
            pad = (1, 1, 0, 0) if halo.axis == 3 else (0, 0, 1, 1)
            y = F.conv2d(F.pad(y, pad), conv.weight, conv.bias)
        else:
            y = conv(y)
        return y.view(b, t, y.shape[1], y.shape[2], y.shape[3]).permute(0, 2, 1, 3, 4)


class MidBlock(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.resnets = nn.ModuleList([ResidualBlock(dim, dim), ResidualBlock(dim, dim)])
        self.attentions = nn.ModuleList([AttentionBlock(dim)])

    def forward(self, x, cache, idx, halo):
        x = self.resnets[0](x, cache, idx, halo)
        x = self.attentions[0](x, halo)
        return self.resnets[1](x, cache, idx, halo)


class UpBlock(nn.Module):
    def __init__(self, cin, cout, blocks, mode):
        super().__init__()
        res = []
        for _ in range(blocks + 1):
            res.append(ResidualBlock(cin, cout))
            cin = cout
        self.resnets = nn.ModuleList(res)
        self.upsamplers = nn.ModuleList([Resample(cout, mode)]) if mode else None

    def forward(self, x, cache, idx, halo):
        for r in self.resnets:
            x = r(x, cache, idx, halo)
        if self.upsamplers is not None:
            x = self.upsamplers[0](x, cache, idx, halo)
        return x


class DupUp3D(nn.Module):
    """Parameter-free shortcut of a Wan2.2 up block: channels repeated, then moved into
    time (factor_t) and space (factor_s x factor_s); the first chunk drops the leading
    duplicated frames (as the causal time upsampler does)."""

    def __init__(self, cin, cout, factor_t, factor_s=1):
        super().__init__()
        self.cout, self.ft, self.fs = cout, factor_t, factor_s
        factor = factor_t * factor_s * factor_s
        if (cout * factor) % cin:
            raise ValueError("DupUp3D: cout * factor must be a multiple of cin")
        self.repeats = cout * factor // cin

    def forward(self, x, first_chunk=False):
        b, _, t, h, w = x.shape
        x = x.repeat_interleave(self.repeats, dim=1)
        x = x.view(b, self.cout, self.ft, self.fs, self.fs, t, h, w)
        x = x.permute(0, 1, 5, 2, 6, 3, 7, 4).reshape(b, self.cout, t * self.ft, h * self.fs, w * self.fs)
        return x[:, :, self.ft - 1:] if first_chunk else x


class ResidualUpBlock(nn.Module):
    """Wan2.2 up block: resnets, optional up-sampler to the same width, plus a DupUp3D
    shortcut of the block input."""

    def __init__(self, cin, cout, blocks, temporal_up, up):
        super().__init__()
        self.avg_shortcut = DupUp3D(cin, cout, 2 if temporal_up else 1, 2) if up else None
        res = []
        c = cin
        for _ in range(blocks + 1):
            res.append(ResidualBlock(c, cout))
            c = cout
        self.resnets = nn.ModuleList(res)
        self.upsampler = Resample(cout, "upsample3d" if temporal_up else "upsample2d", out_dim=cout) if up else None

    def forward(self, x, cache, idx, halo, first_chunk=False):
        x_in = x
        for r in self.resnets:
            x = r(x, cache, idx, halo)
        if self.upsampler is not None:
            x = self.upsampler(x, cache, idx, halo)
        if self.avg_shortcut is not None:
            x = x + self.avg_shortcut(x_in, first_chunk=first_chunk)
        return x


class Decoder3d(nn.Module):
    def __init__(self, dim=96, z_dim=16, mult=(1, 2, 4, 4), blocks=2, temporal_up=(True, True, False),
                 out_channels=3, residual=False):
        super().__init__()
        dims = [dim * m for m in [mult[-1]] + list(mult[::-1])]
        self.residual = residual
        self.conv_in = CausalConv3d(z_dim, dims[0], 3, padding=1)
        self.mid_block = MidBlock(dims[0])
        ups = []
        for i, (cin, cout) in enumerate(zip(dims[:-1], dims[1:])):
            up = i != len(mult) - 1
            if residual:
                ups.append(ResidualUpBlock(cin, cout, blocks, temporal_up[i] if up else False, up))
                continue
            if i > 0:
                cin //= 2
            mode = None
            if up:
                mode = "upsample3d" if temporal_up[i] else "upsample2d"
            ups.append(UpBlock(cin, cout, blocks, mode))
        self.up_blocks = nn.ModuleList(ups)
        self.norm_out = RMSNormC(dims[-1], images=False)
        self.conv_out = CausalConv3d(dims[-1], out_channels, 3, padding=1)

    def forward(self, x, cache, idx, halo, first_chunk=False):
        new = x[:, :, -CACHE_T:].clone()
        x = self.conv_in(x, cache[idx[0]], halo)
        cache[idx[0]] = new
        idx[0] += 1
        x = self.mid_block(x, cache, idx, halo)
        for up in self.up_blocks:
            x = up(x, cache, idx, halo, first_chunk) if self.residual else up(x, cache, idx, halo)
        x = F.silu(self.norm_out(x))
        new = x[:, :, -CACHE_T:].clone()
        old = cache[idx[0]]
        if new.shape[2] < 2 and old is not None:
            new = torch.cat([old[:, :, -1:].to(new.device), new], dim=2)
        x = self.conv_out(x, old, halo)
        cache[idx[0]] = new
        idx[0] += 1
        return x


class WanVAEDecoder(nn.Module):
    """``variant``: "wan2.1" (z 16, base 96, 8x spatial) or "wan2.2" (z 48, decoder base 256,
    residual up blocks, 12 channels un-patchified 2x2: 16x spatial).  Latent statistics
    default to the Wan2.1 values, or zero mean / unit std for Wan2.2 until a checkpoint's
    config provides them (``set_latent_stats``)."""

    VARIANTS = {"wan2.1": dict(z_dim=16, base=96, residual=False, patch=1),
                "wan2.2": dict(z_dim=48, base=256, residual=True, patch=2)}

    def __init__(self, z_dim=16, base=96, residual=False, patch=1):
        super().__init__()
        self.z_dim, self.patch = z_dim, patch
        self.post_quant_conv = CausalConv3d(z_dim, z_dim, 1)
        self.decoder = Decoder3d(base, z_dim, out_channels=3 * patch * patch, residual=residual)
        mean = WAN21_LATENTS_MEAN if z_dim == 16 else [0.0] * z_dim
        std = WAN21_LATENTS_STD if z_dim == 16 else [1.0] * z_dim
        self.register_buffer("latents_mean", torch.tensor(mean).view(1, z_dim, 1, 1, 1))
        self.register_buffer("latents_std", torch.tensor(std).view(1, z_dim, 1, 1, 1))

    @classmethod
    def random_init(cls, device="cpu", dtype=torch.bfloat16, seed: int = 0, variant: str = "wan2.1") -> "WanVAEDecoder":
        torch.manual_seed(seed)
        m = cls(**cls.VARIANTS[variant]).to(device)
        return m.to(dtype).eval()

    def set_latent_stats(self, mean, std):
        self.latents_mean.copy_(torch.tensor(mean).view_as(self.latents_mean))
        self.latents_std.copy_(torch.tensor(std).view_as(self.latents_std))

    def cache_size(self) -> int:
        return sum(isinstance(m, CausalConv3d) for m in self.decoder.modules())

    @torch.inference_mode()
    def decode_frame(self, z_frame: torch.Tensor, cache: list, halo: Halo | None = None,
                     first_chunk: bool = False) -> torch.Tensor:
        """Decode one latent frame [B, C, 1, h, w] (already de-normalised), updating ``cache``."""
        halo = halo or Halo()
        x = self.post_quant_conv(z_frame)
        idx = [0]
        out = self.decoder(x, cache, idx, halo, first_chunk)
        return self.unpatchify(out)

    def unpatchify(self, x: torch.Tensor) -> torch.Tensor:
        """[B, 3 p p, T, H, W] -> [B, 3, T, H p, W p] (channel = c p p + r p + q; q along H)."""
        p = self.patch
        if p == 1:
            return x
        b, cpp, t, h, w = x.shape
        c = cpp // (p * p)
        return x.view(b, c, p, p, t, h, w).permute(0, 1, 4, 5, 3, 6, 2).reshape(b, c, t, h * p, w * p)

    def denormalize(self, z: torch.Tensor) -> torch.Tensor:
        return z * self.latents_std.to(z) + self.latents_mean.to(z)

    @torch.inference_mode()
    def decode(self, z: torch.Tensor, halo: Halo | None = None) -> torch.Tensor:
        """[B, z, F, h, w] normalised latents -> [B, 3, 1 + 4(F-1), s h, s w] in [-1, 1]."""
        dec = ChunkedDecode(self, z, halo)
        while not dec.done:
            dec.step()
        return dec.result()


class ChunkedDecode:
    """Resumable per-latent-frame decode (pause between frames, identical result)."""

    def __init__(self, vae: WanVAEDecoder, z: torch.Tensor, halo: Halo | None = None):
        self.vae = vae
        self.z = vae.denormalize(z.to(next(vae.parameters()).dtype))
        self.halo = halo or Halo()
        self.cache = [None] * 64
        self.next = 0
        self.frames: list = []

    @property
    def done(self) -> bool:
        return self.next >= self.z.shape[2]

    def step(self, frames: int = 1):
        for _ in range(frames):
            if self.done:
                break
            i = self.next
            out = self.vae.decode_frame(self.z[:, :, i:i + 1], self.cache, self.halo, first_chunk=i == 0)
            self.frames.append(out.clamp(-1, 1))
            self.next += 1
        return self

    def result(self) -> torch.Tensor:
        return torch.cat(self.frames, dim=2)


class PatchParallel(Halo):
    """Spatial split over a process group along H (axis 3) or W (axis 4).

    ``pad`` exchanges one boundary slice with each neighbour (torch.distributed send/recv,
    the baseline transport; ``parallel.fused`` swaps in peer-memory stores) and returns the
    local slab with a halo on each side (zeros at the frame edge); ``gather`` all-gathers a
    feature map along the split axis (mid-block attention); ``local`` cuts this rank's part.
    """

    def __init__(self, group=None, axis: int = 4):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.axis = axis
        self.ranks = dist.get_process_group_ranks(group) if group is not None else list(range(self.size))

    def pad(self, x):
        d = self.dist
        a = self.axis
        n = x.shape[a]
        first = x.narrow(a, 0, 1).contiguous()
        last = x.narrow(a, n - 1, 1).contiguous()
        left = torch.zeros_like(first)
        right = torch.zeros_like(last)
        ops = []
        if self.rank > 0:
            peer = self.ranks[self.rank - 1]
            ops += [d.P2POp(d.isend, first, peer, self.group), d.P2POp(d.irecv, left, peer, self.group)]
        if self.rank < self.size - 1:
            peer = self.ranks[self.rank + 1]
            ops += [d.P2POp(d.isend, last, peer, self.group), d.P2POp(d.irecv, right, peer, self.group)]
        if ops:
            for w in d.batch_isend_irecv(ops):
                w.wait()
        return torch.cat([left, x, right], dim=a)

    def gather(self, x):
        parts = [torch.empty_like(x) for _ in range(self.size)]
        self.dist.all_gather(parts, x.contiguous(), group=self.group)
        return torch.cat(parts, dim=self.axis)

    def local(self, x):
        n = x.shape[self.axis] // self.size
        return x.narrow(self.axis, self.rank * n, n)


def split_latent(z: torch.Tensor, halo: Halo) -> torch.Tensor:
    """This rank's slab of a full latent along the halo's split axis."""
    if halo.size == 1:
        return z
    n = z.shape[halo.axis]
    if n % halo.size:
        raise ValueError(f"latent axis of {n} does not split over {halo.size} ranks")
    return z.narrow(halo.axis, halo.rank * (n // halo.size), n // halo.size).contiguous()
