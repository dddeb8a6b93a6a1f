"""SD3.5-Medium MMDiT on the sm_100a ops, with token-packed heterogeneous batches.

Parameter names follow diffusers ``SD3Transformer2DModel`` (pos_embed.proj, time_text_embed.*,
context_embedder, transformer_blocks.i.{norm1, norm1_context, attn, attn2, ff, ff_context},
norm_out.linear, proj_out) so a diffusers/safetensors checkpoint loads with ``load_state_dict``.

Packed layout (one step of a continuous batch of R segments — requests x CFG branches):
  X = [ image tokens of segment 0 .. R-1 | text tokens of segment 0 .. R-1 ]   rows of one buffer
Each segment's joint attention runs over (its image range, its text range) via the dual-range
segment table of ``ops.attention_segments``; no joint sequence is ever concatenated.  Modulation
is per segment through a row -> segment map (``row_batch``) in the LN-modulate kernel and the
gated-residual GEMM epilogue.  Different resolutions in one batch cost only their own tokens.
Reference: workers/ditserve/models/sd35_batch.py:135-736 (packed adaLN-Zero, varlen joint
attention, per-segment unpatchify), sd35.py:816-1164 (continuous batching).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
from torch import nn

from ... import ops
from ..wan.model import Linear, RMSWeight, timestep_sinusoid


@dataclass(frozen=True)
class SD35Config:
    name: str = "sd3.5-medium"
    layers: int = 24
    heads: int = 24
    head_dim: int = 64
    in_channels: int = 16
    out_channels: int = 16
    patch: int = 2
    joint_dim: int = 4096
    pooled_dim: int = 2048
    pos_max: int = 384
    dual_layers: tuple = tuple(range(13))
    eps: float = 1e-6
    ffn_mult: int = 4
    shift: float = 3.0
    vae_scale: int = 8

    @property
    def dim(self) -> int:
        return self.heads * self.head_dim


SD35_MEDIUM = SD35Config()
SD35_TINY = SD35Config(name="sd3.5-tiny", layers=3, heads=4, head_dim=64, joint_dim=256, pooled_dim=128, pos_max=64,
                       dual_layers=(0,))


class _Proj(nn.Module):
    def __init__(self, dim, hidden):
        super().__init__()
        self.proj = Linear(dim, hidden)


class FeedForward(nn.Module):
    def __init__(self, dim, hidden):
        super().__init__()
        self.net = nn.ModuleList([_Proj(dim, hidden), nn.Identity(), Linear(hidden, dim)])


class JointAttention(nn.Module):
    def __init__(self, dim, heads, context: bool, context_pre_only: bool):
        super().__init__()
        hd = dim // heads
        self.to_q, self.to_k, self.to_v = Linear(dim, dim), Linear(dim, dim), Linear(dim, dim)
        self.to_out = nn.ModuleList([Linear(dim, dim)])
        self.norm_q, self.norm_k = RMSWeight(hd), RMSWeight(hd)
        if context:
            self.add_q_proj, self.add_k_proj, self.add_v_proj = Linear(dim, dim), Linear(dim, dim), Linear(dim, dim)
            self.norm_added_q, self.norm_added_k = RMSWeight(hd), RMSWeight(hd)
            if not context_pre_only:
                self.to_add_out = Linear(dim, dim)
        self.register_buffer("w_qkv", None, persistent=False)
        self.register_buffer("b_qkv", None, persistent=False)
        self.register_buffer("w_add_qkv", None, persistent=False)
        self.register_buffer("b_add_qkv", None, persistent=False)

    def fuse(self):
        with torch.no_grad():
            self.w_qkv = torch.cat([self.to_q.weight, self.to_k.weight, self.to_v.weight]).contiguous()
            self.b_qkv = torch.cat([self.to_q.bias, self.to_k.bias, self.to_v.bias]).contiguous()
            if hasattr(self, "add_q_proj"):
                self.w_add_qkv = torch.cat([self.add_q_proj.weight, self.add_k_proj.weight,
                                            self.add_v_proj.weight]).contiguous()
                self.b_add_qkv = torch.cat([self.add_q_proj.bias, self.add_k_proj.bias,
                                            self.add_v_proj.bias]).contiguous()


class AdaLN(nn.Module):
    def __init__(self, dim, chunks):
        super().__init__()
        self.linear = Linear(dim, chunks * dim)
        self.chunks = chunks


class JointBlock(nn.Module):
    def __init__(self, cfg: SD35Config, index: int):
        super().__init__()
        d = cfg.dim
        self.dual = index in cfg.dual_layers
        self.context_pre_only = index == cfg.layers - 1
        self.norm1 = AdaLN(d, 9 if self.dual else 6)
        self.norm1_context = AdaLN(d, 2 if self.context_pre_only else 6)
        self.attn = JointAttention(d, cfg.heads, True, self.context_pre_only)
        if self.dual:
            self.attn2 = JointAttention(d, cfg.heads, False, True)
        self.ff = FeedForward(d, cfg.ffn_mult * d)
        if not self.context_pre_only:
            self.ff_context = FeedForward(d, cfg.ffn_mult * d)


class PosEmbed(nn.Module):
    def __init__(self, cfg: SD35Config):
        super().__init__()
        self.proj_weight_shape = (cfg.dim, cfg.in_channels, cfg.patch, cfg.patch)
        self.proj = nn.Module()
        self.proj.weight = nn.Parameter(torch.empty(*self.proj_weight_shape))
        self.proj.bias = nn.Parameter(torch.empty(cfg.dim))
        self.register_buffer("w2d", None, persistent=False)

    def fuse(self):
        with torch.no_grad():
            self.w2d = self.proj.weight.reshape(self.proj.weight.shape[0], -1).contiguous()


def sincos_2d(dim: int, grid: int) -> np.ndarray:
    """Fixed 2-D sine-cosine position table [grid*grid, dim] (half the channels per axis)."""
    def one_axis(d, pos):
        omega = 1.0 / 10000 ** (np.arange(d // 2, dtype=np.float64) / (d / 2.0))
        out = np.outer(pos.reshape(-1), omega)
        return np.concatenate([np.sin(out), np.cos(out)], axis=1)
    gh, gw = np.meshgrid(np.arange(grid, dtype=np.float64), np.arange(grid, dtype=np.float64), indexing="ij")
    emb_h = one_axis(dim // 2, gh)
    emb_w = one_axis(dim // 2, gw)
    return np.concatenate([emb_w, emb_h], axis=1)


class SD35Transformer(nn.Module):
    def __init__(self, cfg: SD35Config):
        super().__init__()
        self.cfg = cfg
        d = cfg.dim
        self.pos_embed = PosEmbed(cfg)
        self.time_text_embed = nn.Module()
        self.time_text_embed.timestep_embedder = nn.Module()
        self.time_text_embed.timestep_embedder.linear_1 = Linear(256, d)
        self.time_text_embed.timestep_embedder.linear_2 = Linear(d, d)
        self.time_text_embed.text_embedder = nn.Module()
        self.time_text_embed.text_embedder.linear_1 = Linear(cfg.pooled_dim, d)
        self.time_text_embed.text_embedder.linear_2 = Linear(d, d)
        self.context_embedder = Linear(cfg.joint_dim, d)
        self.transformer_blocks = nn.ModuleList([JointBlock(cfg, i) for i in range(cfg.layers)])
        self.norm_out = AdaLN(d, 2)
        self.proj_out = Linear(d, cfg.patch * cfg.patch * cfg.out_channels)
        self._pos_cache: dict = {}

    @classmethod
    def random_init(cls, cfg: SD35Config, device="cpu", dtype=torch.bfloat16, seed: int = 0) -> "SD35Transformer":
        with torch.device("meta"):
            m = cls(cfg)
        m = m.to_empty(device=device)
        gen = torch.Generator(device=device).manual_seed(seed)
        with torch.no_grad():
            for mod in m.modules():
                if isinstance(mod, Linear):
                    mod.reset(gen)
                elif isinstance(mod, RMSWeight):
                    mod.weight.fill_(1.0)
            w = m.pos_embed.proj.weight
            bound = 1.0 / math.sqrt(w[0].numel())
            w.uniform_(-bound, bound, generator=gen)
            m.pos_embed.proj.bias.uniform_(-bound, bound, generator=gen)
        m = m.to(dtype)
        m.prepare()
        m.eval()
        return m

    def prepare(self):
        for blk in self.transformer_blocks:
            blk.attn.fuse()
            if blk.dual:
                blk.attn2.fuse()
        self.pos_embed.fuse()
        return self

    # ------------------------------------------------------------------ helpers
    def pos_table(self, h: int, w: int, device) -> torch.Tensor:
        """Center crop of the pos_max x pos_max sin-cos table for an h x w patch grid."""
        key = (h, w, str(device))
        if key not in self._pos_cache:
            full = sincos_2d(self.cfg.dim, self.cfg.pos_max).reshape(self.cfg.pos_max, self.cfg.pos_max, -1)
            top, left = (self.cfg.pos_max - h) // 2, (self.cfg.pos_max - w) // 2
            crop = full[top:top + h, left:left + w].reshape(h * w, -1)
            self._pos_cache[key] = torch.from_numpy(crop).float().to(device)
        return self._pos_cache[key]

    def patchify(self, lat: torch.Tensor) -> torch.Tensor:
        C, H, W = lat.shape
        p = self.cfg.patch
        x = lat.reshape(C, H // p, p, W // p, p).permute(1, 3, 0, 2, 4)
        return x.reshape((H // p) * (W // p), C * p * p)

    def unpatchify(self, y: torch.Tensor, H: int, W: int) -> torch.Tensor:
        p, C = self.cfg.patch, self.cfg.out_channels
        h, w = H // p, W // p
        return y.reshape(h, w, p, p, C).permute(4, 0, 2, 1, 3).reshape(C, H, W)

    # ------------------------------------------------------------------ packed forward
    @torch.inference_mode()
    def forward_packed(self, latents: list, timesteps: list, contexts: list, pooled: list, cache=None) -> list:
        """One denoising forward of R segments of possibly different resolutions.

        latents[i] [C, H_i, W_i], timesteps[i] float, contexts[i] [L_i, joint_dim], pooled[i] [pooled_dim].
        Returns the velocity predictions [C, H_i, W_i] (model dtype).  ``cache`` (an
        approximate-mode ``BlockResidualCache``) reuses the middle blocks' residual.
        """
        cfg = self.cfg
        dev = self.proj_out.weight.device
        dtype = self.proj_out.weight.dtype
        d, H, hd = cfg.dim, cfg.heads, cfg.head_dim
        R = len(latents)
        img_len = [(l.shape[1] // cfg.patch) * (l.shape[2] // cfg.patch) for l in latents]
        txt_len = [c.shape[0] for c in contexts]
        Ti, Tt = sum(img_len), sum(txt_len)
        T = Ti + Tt
        # segment tables and row -> segment maps
        segs, rb = [], []
        io, to = 0, Ti
        for i in range(R):
            segs.append((io, io + img_len[i], to, to + txt_len[i], io, io + img_len[i], to, to + txt_len[i]))
            io += img_len[i]
            to += txt_len[i]
        row_seg = torch.cat([torch.full((img_len[i],), i, dtype=torch.int32) for i in range(R)] +
                            [torch.full((txt_len[i],), i, dtype=torch.int32) for i in range(R)]).to(dev)
        joint_tbl = ops.segment_table(segs)
        img_tbl = ops.segment_table([(s[0], s[1], 0, 0, s[0], s[1], 0, 0) for s in segs])
        # patch embed + positions (image rows), context embed (text rows)
        x = torch.empty(T, d, device=dev, dtype=dtype)
        patches = torch.cat([self.patchify(l.to(dtype)) for l in latents], 0)
        ops.linear(patches, self.pos_embed.w2d, self.pos_embed.proj.bias, out=x[:Ti])
        pos = torch.cat([self.pos_table(l.shape[1] // cfg.patch, l.shape[2] // cfg.patch, dev) for l in latents], 0)
        x[:Ti] = (x[:Ti].float() + pos).to(dtype)
        ctx = torch.cat([c.to(dev, dtype) for c in contexts], 0)
        ops.linear(ctx, self.context_embedder.weight, self.context_embedder.bias, out=x[Ti:])
        # conditioning: timestep MLP + pooled text MLP
        te = self.time_text_embed
        tsin = timestep_sinusoid(torch.tensor(timesteps, device=dev, dtype=torch.float32), 256).to(dtype)
        h = te.timestep_embedder.linear_1(tsin)
        temb = te.timestep_embedder.linear_2(torch.nn.functional.silu(h.float()).to(dtype))
        pp = torch.stack([p.to(dev, dtype) for p in pooled], 0)
        h = te.text_embedder.linear_1(pp)
        cond = temb.float() + te.text_embedder.linear_2(torch.nn.functional.silu(h.float()).to(dtype)).float()
        cond_act = torch.nn.functional.silu(cond).to(dtype)  # [R, d]
        row_img, row_txt = row_seg[:Ti], row_seg[Ti:]
        blocks = self.transformer_blocks
        if cache is None:
            for blk in blocks:
                x = self._block(blk, x, cond_act, Ti, Tt, row_img, row_txt, joint_tbl, img_tbl)
        else:
            x = cache.run_blocks(lambda i, h: self._block(blocks[i], h, cond_act, Ti, Tt, row_img, row_txt, joint_tbl,
                                                          img_tbl), x, key=(tuple(img_len), tuple(txt_len)))
        # final adaLN-continuous (scale first, then shift) + projection, image rows only
        emb = self.norm_out.linear(cond_act).float()
        scale, shift = emb[:, :d], emb[:, d:]
        hn = ops.layernorm_modulate(x[:Ti], scale=scale, shift=shift, eps=cfg.eps, row_batch=row_img)
        y = ops.linear(hn, self.proj_out.weight, self.proj_out.bias)
        out, off = [], 0
        for i, l in enumerate(latents):
            out.append(self.unpatchify(y[off:off + img_len[i]], l.shape[1], l.shape[2]))
            off += img_len[i]
        return out

    def _block(self, blk: JointBlock, x, cond_act, Ti, Tt, row_img, row_txt, joint_tbl, img_tbl):
        cfg = self.cfg
        d, H = cfg.dim, cfg.heads
        xi, xt = x[:Ti], x[Ti:]
        m = blk.norm1.linear(cond_act).float()        # [R, (6|9) d]
        mc = blk.norm1_context.linear(cond_act).float()  # [R, (2|6) d]
        sh_msa, sc_msa, g_msa, sh_mlp, sc_mlp, g_mlp = (m[:, i * d:(i + 1) * d] for i in range(6))
        hi = ops.layernorm_modulate(xi, scale=sc_msa, shift=sh_msa, eps=cfg.eps, row_batch=row_img)
        h2 = None
        if blk.dual:
            # second modulation of the same normalised input (before any residual update)
            sh2, sc2, g2 = (m[:, i * d:(i + 1) * d] for i in range(6, 9))
            h2 = ops.layernorm_modulate(xi, scale=sc2, shift=sh2, eps=cfg.eps, row_batch=row_img)
        if blk.context_pre_only:
            ht = ops.layernorm_modulate(xt, scale=mc[:, :d], shift=mc[:, d:], eps=cfg.eps, row_batch=row_txt)
        else:
            c_sh_msa, c_sc_msa, c_g_msa, c_sh_mlp, c_sc_mlp, c_g_mlp = (mc[:, i * d:(i + 1) * d] for i in range(6))
            ht = ops.layernorm_modulate(xt, scale=c_sc_msa, shift=c_sh_msa, eps=cfg.eps, row_batch=row_txt)
        a = blk.attn
        qkv = torch.empty(Ti + Tt, 3 * d, device=x.device, dtype=x.dtype)
        ops.linear(hi, a.w_qkv, a.b_qkv, out=qkv[:Ti])
        ops.linear(ht, a.w_add_qkv, a.b_add_qkv, out=qkv[Ti:])
        for part, (wi, wt) in enumerate(((a.norm_q, a.norm_added_q), (a.norm_k, a.norm_added_k))):
            ops.rmsnorm_rope_(qkv[:Ti, part * d:(part + 1) * d], wi.weight, groups=H, eps=cfg.eps, head_dim=cfg.head_dim)
            ops.rmsnorm_rope_(qkv[Ti:, part * d:(part + 1) * d], wt.weight, groups=H, eps=cfg.eps, head_dim=cfg.head_dim)
        o = ops.attention_segments(qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:], H, joint_tbl)
        xi = ops.linear(o[:Ti], a.to_out[0].weight, a.to_out[0].bias, residual=xi, gate=g_msa, row_batch=row_img,
                        out=xi if xi.is_cuda else None)
        if blk.dual:
            a2 = blk.attn2
            qkv2 = ops.linear(h2, a2.w_qkv, a2.b_qkv)
            ops.rmsnorm_rope_(qkv2[:, :d], a2.norm_q.weight, groups=H, eps=cfg.eps, head_dim=cfg.head_dim)
            ops.rmsnorm_rope_(qkv2[:, d:2 * d], a2.norm_k.weight, groups=H, eps=cfg.eps, head_dim=cfg.head_dim)
            o2 = ops.attention_segments(qkv2[:, :d], qkv2[:, d:2 * d], qkv2[:, 2 * d:], H, img_tbl)
            xi = ops.linear(o2, a2.to_out[0].weight, a2.to_out[0].bias, residual=xi, gate=g2, row_batch=row_img,
                            out=xi if xi.is_cuda else None)
        hi = ops.layernorm_modulate(xi, scale=sc_mlp, shift=sh_mlp, eps=cfg.eps, row_batch=row_img)
        f = ops.linear(hi, blk.ff.net[0].proj.weight, blk.ff.net[0].proj.bias, act="gelu")
        xi = ops.linear(f, blk.ff.net[2].weight, blk.ff.net[2].bias, residual=xi, gate=g_mlp, row_batch=row_img,
                        out=xi if xi.is_cuda else None)
        if not blk.context_pre_only:
            xt = ops.linear(o[Ti:], a.to_add_out.weight, a.to_add_out.bias, residual=xt, gate=c_g_msa,
                            row_batch=row_txt, out=xt if xt.is_cuda else None)
            ht = ops.layernorm_modulate(xt, scale=c_sc_mlp, shift=c_sh_mlp, eps=cfg.eps, row_batch=row_txt)
            f = ops.linear(ht, blk.ff_context.net[0].proj.weight, blk.ff_context.net[0].proj.bias, act="gelu")
            xt = ops.linear(f, blk.ff_context.net[2].weight, blk.ff_context.net[2].bias, residual=xt, gate=c_g_mlp,
                            row_batch=row_txt, out=xt if xt.is_cuda else None)
        if x.is_cuda:
            return x  # residual updates were written in place into the packed buffer
        return torch.cat([xi, xt], 0)
