"""Channels-last decode of the Wan VAE on the implicit-GEMM tcgen05 convolution.

``FastDecoder(vae)`` runs the same module (same parameters, same causal frame cache, same
per-latent-frame schedule as ``vae.ChunkedDecode``) with activations laid out [T, H, W, C]
so every 3x3x3, 1x3x3, 3x1x1 and 1x1x1 convolution is one ``ops.conv_cl`` launch (spatial
zero padding by the kernel's TMA out-of-bounds fill, the residual add of a block fused into
its second conv's epilogue).  Norms, SiLU and the nearest upsampling are channels-last torch
ops; the mid-block attention (one head of 384 channels at latent resolution) uses torch SDPA.

Patch parallelism: with a halo (``HaloCL``) the frame is split along H; before every conv
with a 3-high kernel the slab is completed with one row from each neighbour and the conv runs
with pad_h = 0, reading only this rank's memory.  The mid-block attention gathers the small
latent-resolution map over the group.

Reference: diffusers AutoencoderKLWan as decoded by the reference's pipeline
(workers/ditserve/models/pipeline.py:171-231) and its distvae patch parallelism
(workers/xfuser/model_executor/pipelines/base_pipeline.py:61,133).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ... import ops
from . import vae as V


class HaloCL:
    """No split (one rank); subclasses exchange boundary rows of [T, H, W, C] slabs."""

    size = 1
    rank = 0

    def pad_rows(self, x: torch.Tensor) -> torch.Tensor:
        return x

    def gather_rows(self, x: torch.Tensor) -> torch.Tensor:
        return x

    def local_rows(self, x: torch.Tensor) -> torch.Tensor:
        return x


class PeerHaloCL(HaloCL):
    """Row halo over a symmetric heap: the first and last rows of this rank's slab are stored
    straight into the neighbours' halo slots (``strided_put`` over NVLink), one bounded group
    barrier, then the slab is completed locally.  ``gather_rows`` uses the NCCL baseline."""

    def __init__(self, peer_halo, group=None):
        self.ph = peer_halo            # parallel.fused.PeerHalo over the decode group, axis unused
        self.group = group
        self.size, self.rank = peer_halo.size, peer_halo.rank

    def pad_rows(self, x):
        # PeerHalo pads along its axis of a 5-D view; a [T, H, W, C] slab is [1, T, H, W, C] with axis 2
        ph = self.ph
        ph.axis = 2
        return ph.pad(x.unsqueeze(0))[0]

    def gather_rows(self, x):
        import torch.distributed as dist
        parts = [torch.empty_like(x) for _ in range(self.size)]
        dist.all_gather(parts, x.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)

    def local_rows(self, x):
        n = x.shape[1] // self.size
        return x.narrow(1, self.rank * n, n)


class NCCLHaloCL(HaloCL):
    """Row halo through torch.distributed send/recv (the baseline transport; also CPU/Gloo)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist, self.group = dist, group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.ranks = dist.get_process_group_ranks(group) if group is not None else list(range(self.size))

    def pad_rows(self, x):
        d = self.dist
        first, last = x[:, :1].contiguous(), x[:, -1:].contiguous()
        left, right = torch.zeros_like(first), torch.zeros_like(last)
        ops_ = []
        if self.rank > 0:
            peer = self.ranks[self.rank - 1]
            ops_ += [d.P2POp(d.isend, first, peer, self.group), d.P2POp(d.irecv, left, peer, self.group)]
        if self.rank < self.size - 1:
            peer = self.ranks[self.rank + 1]
            ops_ += [d.P2POp(d.isend, last, peer, self.group), d.P2POp(d.irecv, right, peer, self.group)]
        if ops_:
            for w in d.batch_isend_irecv(ops_):
                w.wait()
        return torch.cat([left, x, right], dim=1)

    def gather_rows(self, x):
        parts = [torch.empty_like(x) for _ in range(self.size)]
        self.dist.all_gather(parts, x.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)

    def local_rows(self, x):
        n = x.shape[1] // self.size
        return x.narrow(1, self.rank * n, n)


def _cl_weights(conv, c_in_pad=None):
    """Kernel-layout weight and padded bias of a conv module, built once and kept on it."""
    key = ("_cl", c_in_pad)
    cached = getattr(conv, "_cl_cache", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    w2d = ops.conv_weight_2d(conv.weight.detach(), c_in_pad=c_in_pad)
    bias = ops.conv_bias(conv.bias.detach(), w2d.shape[0]) if conv.bias is not None else None
    conv._cl_cache = (key, (w2d, bias))
    return w2d, bias


def _ksize(conv):
    k = conv.kernel_size
    return (1, k[0], k[1]) if len(k) == 2 else tuple(k)


class FastDecoder:
    """Channels-last, per-latent-frame decode of a ``WanVAEDecoder`` (any device: CPU runs the
    convs' fp32 statement)."""

    def __init__(self, vae: V.WanVAEDecoder, halo: HaloCL | None = None):
        self.vae = vae
        self.dec = vae.decoder
        self.halo = halo or HaloCL()

    # ------------------------------------------------------------------ building blocks
    def conv(self, conv, x, cache=None, residual=None):
        """Causal conv on a [T, H, W, C] slab; ``cache`` = the last input frames of the previous
        call (or None on the first chunk, which pads with zero frames)."""
        kt, kh, kw = _ksize(conv)
        c_in = x.shape[-1]
        w2d, bias = _cl_weights(conv, c_in_pad=c_in if c_in % 32 == 0 else None)
        if w2d.shape[1] != kt * kh * kw * c_in:  # channels padded to the kernel's 32-channel step
            x = F.pad(x, (0, w2d.shape[1] // (kt * kh * kw) - c_in))
        tp = getattr(conv, "tpad", 0)
        if tp > 0:
            if cache is not None:
                cache = cache.to(x.dtype)
                if cache.shape[-1] != x.shape[-1]:
                    cache = F.pad(cache, (0, x.shape[-1] - cache.shape[-1]))
                x = torch.cat([cache, x], dim=0)
                tp -= cache.shape[0]
            if tp > 0:
                x = torch.cat([x.new_zeros((tp,) + tuple(x.shape[1:])), x], dim=0)
        ph = (kh - 1) // 2
        pw = (kw - 1) // 2
        if self.halo.size > 1 and ph > 0:
            x = self.halo.pad_rows(x)
            ph = 0
        c_out = conv.weight.shape[0]
        return ops.conv_cl(x.contiguous(), w2d, bias, (kt, kh, kw), (ph, pw), c_out, residual=residual)

    @staticmethod
    def norm(mod, x):
        y = F.normalize(x.float(), dim=-1) * mod.scale * mod.gamma.float().reshape(-1)
        if mod.bias is not None:
            y = y + mod.bias.float().reshape(-1)
        return y.to(x.dtype)

    def _cached_conv(self, conv, x, cache, idx, residual=None):
        new = x[-V.CACHE_T:].clone()
        old = cache[idx[0]]
        if new.shape[0] < 2 and old is not None:
            new = torch.cat([old[-1:].to(new.device), new], dim=0)
        out = self.conv(conv, x, old, residual=residual)
        cache[idx[0]] = new
        idx[0] += 1
        return out

    def resblock(self, blk, x, cache, idx):
        h = self.conv(blk.conv_shortcut, x) if blk.conv_shortcut is not None else x
        x = F.silu(self.norm(blk.norm1, x))
        x = self._cached_conv(blk.conv1, x, cache, idx)
        x = F.silu(self.norm(blk.norm2, x))
        return self._cached_conv(blk.conv2, x, cache, idx, residual=h.contiguous())

    def attention(self, blk, x):
        identity = x
        full = self.halo.gather_rows(x)
        t, h, w, c = full.shape
        y = self.norm(blk.norm, full).reshape(t * h * w, c)
        qkv = ops.linear(y, blk.to_qkv.weight.reshape(3 * c, c), blk.to_qkv.bias)
        q, k, v = qkv.reshape(t, h * w, 3, c).unbind(2)
        o = F.scaled_dot_product_attention(q.unsqueeze(1), k.unsqueeze(1), v.unsqueeze(1)).squeeze(1)
        o = ops.linear(o.reshape(t * h * w, c), blk.proj.weight.reshape(c, c), blk.proj.bias).reshape(t, h, w, c)
        return self.halo.local_rows(o) + identity

    @staticmethod
    def up2(x):
        t, h, w, c = x.shape
        return x[:, :, None, :, None, :].expand(t, h, 2, w, 2, c).reshape(t, 2 * h, 2 * w, c)

    def resample(self, mod, x, cache, idx):
        if mod.mode == "upsample3d":
            i = idx[0]
            if cache[i] is None:
                cache[i] = "first"  # the first latent frame is not doubled in time
                idx[0] += 1
            else:
                new = x[-V.CACHE_T:].clone()
                if new.shape[0] < 2 and isinstance(cache[i], torch.Tensor):
                    new = torch.cat([cache[i][-1:].to(new.device), new], dim=0)
                if new.shape[0] < 2 and isinstance(cache[i], str):
                    new = torch.cat([torch.zeros_like(new), new], dim=0)
                old = None if isinstance(cache[i], str) else cache[i]
                y = self.conv(mod.time_conv, x, old)
                cache[i] = new
                idx[0] += 1
                t, h, w, c2 = y.shape
                c = c2 // 2
                x = y.reshape(t, h, w, 2, c).permute(0, 3, 1, 2, 4).reshape(2 * t, h, w, c)
        return self.conv(mod.resample[1], self.up2(x))

    def dup_up(self, mod, x, first_chunk):
        t, h, w, _ = x.shape
        y = x.repeat_interleave(mod.repeats, dim=-1)
        y = y.reshape(t, h, w, mod.cout, mod.ft, mod.fs, mod.fs)
        # channel (c, ft, fh, fw) -> frame t * ft + ft_i, row h * fs + fh, column w * fs + fw
        y = y.permute(0, 4, 1, 5, 2, 6, 3).reshape(t * mod.ft, h * mod.fs, w * mod.fs, mod.cout)
        return y[mod.ft - 1:] if first_chunk else y

    # ------------------------------------------------------------------ one latent frame
    @torch.inference_mode()
    def decode_frame(self, z_frame: torch.Tensor, cache: list, first_chunk: bool = False) -> torch.Tensor:
        """[1, z, 1, h, w] de-normalised latent frame (this rank's rows) -> [1, C_out, T, H, W]."""
        d = self.dec
        x = z_frame[0].permute(1, 2, 3, 0).contiguous()  # [1, h, w, z]
        x = self.conv(self.vae.post_quant_conv, x)
        idx = [0]
        new = x[-V.CACHE_T:].clone()  # conv_in keeps the raw last frames (no carry-over of older ones)
        x = self.conv(d.conv_in, x, cache[idx[0]])
        cache[idx[0]] = new
        idx[0] += 1
        mb = d.mid_block
        x = self.resblock(mb.resnets[0], x, cache, idx)
        x = self.attention(mb.attentions[0], x)
        x = self.resblock(mb.resnets[1], x, cache, idx)
        for up in d.up_blocks:
            if d.residual:
                x_in = x
                for r in up.resnets:
                    x = self.resblock(r, x, cache, idx)
                if up.upsampler is not None:
                    x = self.resample(up.upsampler, x, cache, idx)
                if up.avg_shortcut is not None:
                    x = x + self.dup_up(up.avg_shortcut, x_in, first_chunk)
            else:
                for r in up.resnets:
                    x = self.resblock(r, x, cache, idx)
                if up.upsamplers is not None:
                    x = self.resample(up.upsamplers[0], x, cache, idx)
        x = F.silu(self.norm(d.norm_out, x))
        x = self._cached_conv(d.conv_out, x, cache, idx)
        out = x.permute(3, 0, 1, 2).unsqueeze(0)  # [1, C, T, H, W]
        return self.vae.unpatchify(out)

    @torch.inference_mode()
    def decode(self, z: torch.Tensor) -> torch.Tensor:
        """[1, z, F, h, w] normalised latents (this rank's rows) -> [1, 3, 1 + 4(F-1), H, W]."""
        dtype = next(self.vae.parameters()).dtype
        zz = self.vae.denormalize(z.to(dtype))
        cache: list = [None] * 64
        frames = []
        for i in range(zz.shape[2]):
            out = self.decode_frame(zz[:, :, i:i + 1], cache, first_chunk=i == 0)
            frames.append(out.clamp(-1, 1))
        return torch.cat(frames, dim=2)


class FastChunkedDecode:
    """``vae.ChunkedDecode`` on the channels-last path: resumable after any latent frame with
    an identical result.  Under a halo, ``z`` is the full latent; this rank decodes its rows
    and ``result`` gathers the group's rows (every rank gets the whole video)."""

    def __init__(self, vae: V.WanVAEDecoder, z: torch.Tensor, halo: HaloCL | None = None):
        self.halo = halo or HaloCL()
        self.fd = FastDecoder(vae, self.halo)
        dtype = next(vae.parameters()).dtype
        zz = vae.denormalize(z.to(dtype))
        if self.halo.size > 1:
            rows = zz.shape[3]
            if rows % self.halo.size:
                raise ValueError(f"latent height {rows} does not split over {self.halo.size} ranks")
            n = rows // self.halo.size
            zz = zz[:, :, :, self.halo.rank * n:(self.halo.rank + 1) * n].contiguous()
        self.z = zz
        self.cache: list = [None] * 64
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
            out = self.fd.decode_frame(self.z[:, :, i:i + 1], self.cache, first_chunk=i == 0)
            self.frames.append(out.clamp(-1, 1))
            self.next += 1
        return self

    def result(self) -> torch.Tensor:
        video = torch.cat(self.frames, dim=2)  # [1, 3, T, H_local, W]
        if self.halo.size > 1:
            rows = self.halo.gather_rows(video[0].permute(1, 2, 3, 0).contiguous())  # [T, H, W, 3]
            video = rows.permute(3, 0, 1, 2).unsqueeze(0)
        return video
