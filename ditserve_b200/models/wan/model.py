"""Wan diffusion transformer on the sm_100a ops.

Parameter names follow the diffusers ``WanTransformer3DModel`` layout so a
diffusers/safetensors checkpoint loads with ``load_state_dict``; the module is
our own and its forward is split the way the block executor needs it:

    packet = model.begin(latents, timestep, context, pctx)   # patch embed, RoPE, conditions
    model.forward_block(i, packet, pctx)                       # one transformer block (in place)
    pred = model.predict(packet, pctx)                         # norm_out, proj_out, gather, unpatchify

(reference split: workers/xfuser/model_executor/models/transformers/transformer_wan.py:307-395).
Hot path per block: fused LN+modulate -> QKV GEMM -> RMS qk-norm+RoPE -> attention (local or
sequence-parallel through ``pctx``) -> out-proj GEMM with the gated-residual epilogue -> affine LN ->
cross-attention -> out-proj with residual epilogue -> LN+modulate -> FFN up GEMM with GELU epilogue ->
FFN down GEMM with gated-residual epilogue.  CPU tensors run the fp32 reference statement of every op.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import nn

from ... import ops
from .config import WanConfig


class Linear(nn.Module):
    def __init__(self, fan_in: int, fan_out: int, bias: bool = True):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(fan_out, fan_in))
        self.bias = nn.Parameter(torch.empty(fan_out)) if bias else None

    def reset(self, gen: torch.Generator | None = None):
        bound = 1.0 / math.sqrt(self.weight.shape[1])
        with torch.no_grad():
            self.weight.uniform_(-bound, bound, generator=gen)
            if self.bias is not None:
                self.bias.uniform_(-bound, bound, generator=gen)

    def forward(self, x, **kw):
        return ops.linear(x, self.weight, self.bias, **kw)


class RMSWeight(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))


class LNAffine(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.bias = nn.Parameter(torch.zeros(dim))


class WanAttention(nn.Module):
    def __init__(self, dim: int, kv_dim: int | None = None):
        super().__init__()
        kv_dim = kv_dim or dim
        self.to_q = Linear(dim, dim)
        self.to_k = Linear(kv_dim, dim)
        self.to_v = Linear(kv_dim, dim)
        self.to_out = nn.ModuleList([Linear(dim, dim)])
        self.norm_q = RMSWeight(dim)
        self.norm_k = RMSWeight(dim)
        self.register_buffer("w_qkv", None, persistent=False)
        self.register_buffer("b_qkv", None, persistent=False)
        self.register_buffer("w_kv", None, persistent=False)
        self.register_buffer("b_kv", None, persistent=False)

    def fuse(self):
        with torch.no_grad():
            self.w_qkv = torch.cat([self.to_q.weight, self.to_k.weight, self.to_v.weight], 0).contiguous()
            self.b_qkv = torch.cat([self.to_q.bias, self.to_k.bias, self.to_v.bias], 0).contiguous()
            self.w_kv = torch.cat([self.to_k.weight, self.to_v.weight], 0).contiguous()
            self.b_kv = torch.cat([self.to_k.bias, self.to_v.bias], 0).contiguous()


class FeedForward(nn.Module):
    """diffusers FeedForward(gelu-approximate) names: net.0.proj, net.2."""

    def __init__(self, dim: int, hidden: int):
        super().__init__()

        class _Proj(nn.Module):
            def __init__(self):
                super().__init__()
                self.proj = Linear(dim, hidden)

        self.net = nn.ModuleList([_Proj(), nn.Identity(), Linear(hidden, dim)])


class WanBlock(nn.Module):
    def __init__(self, cfg: WanConfig):
        super().__init__()
        d = cfg.dim
        self.attn1 = WanAttention(d)
        self.attn2 = WanAttention(d)
        self.norm2 = LNAffine(d)
        self.ffn = FeedForward(d, cfg.ffn_dim)
        self.scale_shift_table = nn.Parameter(torch.randn(1, 6, d) / d ** 0.5)


class TimeEmbedding(nn.Module):
    def __init__(self, freq_dim: int, dim: int):
        super().__init__()
        self.linear_1 = Linear(freq_dim, dim)
        self.linear_2 = Linear(dim, dim)


class TextProjection(nn.Module):
    def __init__(self, text_dim: int, dim: int):
        super().__init__()
        self.linear_1 = Linear(text_dim, dim)
        self.linear_2 = Linear(dim, dim)


class ConditionEmbedder(nn.Module):
    def __init__(self, cfg: WanConfig):
        super().__init__()
        self.time_embedder = TimeEmbedding(cfg.freq_dim, cfg.dim)
        self.time_proj = Linear(cfg.dim, 6 * cfg.dim)
        self.text_embedder = TextProjection(cfg.text_dim, cfg.dim)


class PatchEmbedding(nn.Module):
    """Conv3d(kernel = stride = patch) stored in its diffusers shape; run as a GEMM."""

    def __init__(self, cfg: WanConfig):
        super().__init__()
        pt, ph, pw = cfg.patch
        self.weight = nn.Parameter(torch.empty(cfg.dim, cfg.in_channels, pt, ph, pw))
        self.bias = nn.Parameter(torch.empty(cfg.dim))
        self.register_buffer("w2d", None, persistent=False)

    def fuse(self):
        with torch.no_grad():
            self.w2d = self.weight.reshape(self.weight.shape[0], -1).contiguous()


def timestep_sinusoid(t: torch.Tensor, dim: int) -> torch.Tensor:
    """[cos | sin] embedding of t (flip_sin_to_cos, shift 0, max period 1e4), fp32."""
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    arg = t.float()[..., None] * freqs
    return torch.cat([torch.cos(arg), torch.sin(arg)], dim=-1)


def rope_tables(cfg: WanConfig, grid: tuple[int, int, int], device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [F*H*W, head_dim/2] for the 3D rotary embedding (t, h, w axes)."""
    d = cfg.head_dim
    dh = dw = 2 * (d // 6)
    dt = d - dh - dw
    f, h, w = grid

    def axis(dim, n):
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
        return torch.outer(torch.arange(n, dtype=torch.float64), inv)  # [n, dim/2]

    at, ah, aw = axis(dt, f), axis(dh, h), axis(dw, w)
    ang = torch.cat([
        at[:, None, None, :].expand(f, h, w, -1),
        ah[None, :, None, :].expand(f, h, w, -1),
        aw[None, None, :, :].expand(f, h, w, -1),
    ], dim=-1).reshape(f * h * w, d // 2)
    return ang.cos().float().to(device).contiguous(), ang.sin().float().to(device).contiguous()


@dataclass
class WanPacket:
    """Continuation state between blocks of one forward (all on device)."""
    x: torch.Tensor            # [B * S_local, D] bf16 hidden states (this rank's sequence shard)
    mod: torch.Tensor          # [B, 6, D] or [B * S_local, 6, D] fp32 timestep projection
    temb: torch.Tensor         # [B, D] or [B * S_local, D] fp32
    ctx: torch.Tensor          # [B * L, D] bf16 projected text context
    cos: torch.Tensor
    sin: torch.Tensor
    batch: int
    seq_local: int
    seq: int
    grid: tuple
    text_len: int
    next_block: int = 0
    cos_full: torch.Tensor | None = None   # whole-sequence tables (fused SP kernels use global positions)
    sin_full: torch.Tensor | None = None

    def tensors(self) -> dict:
        return dict(x=self.x, mod=self.mod, temb=self.temb, ctx=self.ctx, cos=self.cos, sin=self.sin)


class LocalAttention:
    """Single-rank attention (SP1)."""

    sp_size = 1
    sp_rank = 0

    def self_attention(self, q, k, v, heads, batch, seq_local):
        return _uniform_attention(q, k, v, heads, batch)

    def self_attention_qkv(self, qkv, heads, batch, seq_local):
        d = qkv.shape[1] // 3
        return _uniform_attention(qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:], heads, batch)

    def gather_sequence(self, x, batch, seq_local):
        return x


def _uniform_attention(q, k, v, heads, batch):
    """q/k/v: [batch * S, H * D] (possibly strided column views of the fused QKV buffer)."""
    t, tk, w = q.shape[0] // batch, k.shape[0] // batch, q.shape[-1]
    o = ops.attention(q.view(batch, t, w), k.view(batch, tk, -1), v.view(batch, tk, -1), heads)
    return o.reshape(batch * t, w)


class WanTransformer(nn.Module):
    def __init__(self, cfg: WanConfig):
        super().__init__()
        self.cfg = cfg
        self.patch_embedding = PatchEmbedding(cfg)
        self.condition_embedder = ConditionEmbedder(cfg)
        self.blocks = nn.ModuleList([WanBlock(cfg) for _ in range(cfg.layers)])
        self.proj_out = Linear(cfg.dim, cfg.out_channels * math.prod(cfg.patch))
        self.scale_shift_table = nn.Parameter(torch.randn(1, 2, cfg.dim) / cfg.dim ** 0.5)
        self._rope_cache: dict = {}

    # ------------------------------------------------------------------ construction
    @classmethod
    def random_init(cls, cfg: WanConfig, device="cpu", dtype=torch.bfloat16, seed: int = 0) -> "WanTransformer":
        """Random weights of the architecture (no checkpoint needed), initialised on ``device``."""
        with torch.device("meta"):
            m = cls(cfg)
        m = m.to_empty(device=device)
        gen = torch.Generator(device=device).manual_seed(seed)
        with torch.no_grad():
            for mod in m.modules():
                if isinstance(mod, Linear):
                    mod.reset(gen)
                elif isinstance(mod, (RMSWeight, LNAffine)):
                    mod.weight.fill_(1.0)
                    if isinstance(mod, LNAffine):
                        mod.bias.zero_()
            pe = m.patch_embedding
            bound = 1.0 / math.sqrt(pe.weight[0].numel())
            pe.weight.uniform_(-bound, bound, generator=gen)
            pe.bias.uniform_(-bound, bound, generator=gen)
            for blk in m.blocks:
                blk.scale_shift_table.normal_(generator=gen).div_(cfg.dim ** 0.5)
            m.scale_shift_table.normal_(generator=gen).div_(cfg.dim ** 0.5)
        m = m.to(dtype)
        # adaLN tables stay fp32 like the reference's fp32 modulation arithmetic
        for blk in m.blocks:
            blk.scale_shift_table.data = blk.scale_shift_table.data.float()
        m.scale_shift_table.data = m.scale_shift_table.data.float()
        m.prepare()
        return m

    def prepare(self):
        """Build fused weight views (QKV, cross KV, 2-D patch weight)."""
        for blk in self.blocks:
            blk.attn1.fuse()
            blk.attn2.fuse()
        self.patch_embedding.fuse()
        return self

    # ------------------------------------------------------------------ forward pieces
    def rope(self, grid, device):
        key = (grid, str(device))
        if key not in self._rope_cache:
            self._rope_cache[key] = rope_tables(self.cfg, grid, device)
        return self._rope_cache[key]

    def patchify(self, latents: torch.Tensor) -> torch.Tensor:
        """[B, C, F, H, W] -> [B, F'*H'*W', C*pt*ph*pw] (Conv3d weight order)."""
        B, C, F, H, W = latents.shape
        pt, ph, pw = self.cfg.patch
        x = latents.reshape(B, C, F // pt, pt, H // ph, ph, W // pw, pw)
        x = x.permute(0, 2, 4, 6, 1, 3, 5, 7)
        return x.reshape(B, (F // pt) * (H // ph) * (W // pw), C * pt * ph * pw)

    def unpatchify(self, y: torch.Tensor, grid, batch: int) -> torch.Tensor:
        f, h, w = grid
        pt, ph, pw = self.cfg.patch
        c = self.cfg.out_channels
        y = y.reshape(batch, f, h, w, pt, ph, pw, c).permute(0, 7, 1, 4, 2, 5, 3, 6)
        return y.reshape(batch, c, f * pt, h * ph, w * pw)

    def embed_conditions(self, timestep: torch.Tensor, context: torch.Tensor, dtype):
        """timestep [B] (or [B, S] per token) -> temb fp32, mod fp32 [.., 6, D]; context -> [B*L, D]."""
        ce = self.condition_embedder
        d = self.cfg.dim
        sin = timestep_sinusoid(timestep, self.cfg.freq_dim)
        shape = sin.shape[:-1]
        h = ce.time_embedder.linear_1(sin.reshape(-1, self.cfg.freq_dim).to(dtype))
        h = torch.nn.functional.silu(h.float()).to(dtype)
        temb = ce.time_embedder.linear_2(h)
        proj = ce.time_proj(torch.nn.functional.silu(temb.float()).to(dtype))
        temb = temb.float().reshape(*shape, d)
        mod = proj.float().reshape(*shape, 6, d)
        B, L, _ = context.shape
        c = ce.text_embedder.linear_1(context.reshape(B * L, -1).to(dtype), act="gelu")
        c = ce.text_embedder.linear_2(c)
        return temb, mod, c

    def begin(self, latents: torch.Tensor, timestep: torch.Tensor, context: torch.Tensor, pctx=None) -> WanPacket:
        pctx = pctx or LocalAttention()
        cfg = self.cfg
        dtype = self.proj_out.weight.dtype
        B, C, F, H, W = latents.shape
        pt, ph, pw = cfg.patch
        grid = (F // pt, H // ph, W // pw)
        S = grid[0] * grid[1] * grid[2]
        P = pctx.sp_size
        if S % P != 0:
            raise ValueError(f"sequence of {S} tokens does not split over {P} ranks")
        Sl = S // P
        r = pctx.sp_rank
        patches = self.patchify(latents.to(dtype))[:, r * Sl:(r + 1) * Sl].reshape(B * Sl, -1)
        x = ops.linear(patches, self.patch_embedding.w2d, self.patch_embedding.bias)
        temb, mod, ctx = self.embed_conditions(timestep, context, dtype)
        if timestep.dim() == 2:  # per-token timesteps: keep this rank's rows
            temb = temb[:, r * Sl:(r + 1) * Sl].reshape(B * Sl, -1)
            mod = mod[:, r * Sl:(r + 1) * Sl].reshape(B * Sl, 6, -1)
        cos_full, sin_full = self.rope(grid, latents.device)
        cos, sin = cos_full[r * Sl:(r + 1) * Sl], sin_full[r * Sl:(r + 1) * Sl]
        return WanPacket(x=x.contiguous(), mod=mod.contiguous(), temb=temb.contiguous(), ctx=ctx.contiguous(),
                         cos=cos.contiguous(), sin=sin.contiguous(), batch=B, seq_local=Sl, seq=S, grid=grid,
                         text_len=context.shape[1], cos_full=cos_full, sin_full=sin_full)

    def forward_block(self, i: int, pk: WanPacket, pctx=None) -> WanPacket:
        pctx = pctx or LocalAttention()
        if hasattr(pctx, "begin_block"):
            pctx.begin_block(i)  # plans with per-block settings (FP8 payload layers)
        cfg = self.cfg
        blk = self.blocks[i]
        D, Hh, hd = cfg.dim, cfg.heads, cfg.head_dim
        rpb = 1 if pk.mod.shape[0] != pk.batch else pk.seq_local  # per-token or per-sample modulation
        m = blk.scale_shift_table.float() + pk.mod  # [B or B*S_local, 6, D] fp32
        x = pk.x
        # --- self attention
        h = ops.layernorm_modulate(x, scale=m[:, 1], shift=m[:, 0], eps=cfg.eps, rows_per_batch=rpb)
        a1 = blk.attn1
        qkv = ops.linear(h, a1.w_qkv, a1.b_qkv)
        if hasattr(pctx, "fused_qkv_attention") and qkv.is_cuda:
            # qk-norm + RoPE + all-to-all in one kernel, attention epilogue scatters O back
            o = pctx.fused_qkv_attention(qkv, a1.norm_q.weight, a1.norm_k.weight, cfg.eps, pk.cos_full, pk.sin_full,
                                         Hh, pk.batch, pk.seq_local)
        else:
            # q and k norm + RoPE in one launch over the fused QKV buffer
            ops.rmsnorm_rope_qk_(qkv, a1.norm_q.weight, a1.norm_k.weight, eps=cfg.eps, cos=pk.cos, sin=pk.sin,
                                 rows_per_batch=pk.seq_local, head_dim=hd)
            o = pctx.self_attention_qkv(qkv, Hh, pk.batch, pk.seq_local)
        x = ops.linear(o, a1.to_out[0].weight, a1.to_out[0].bias, residual=x, gate=m[:, 2], rows_per_batch=rpb,
                       out=x if x.is_cuda else None)
        # --- cross attention (no sequence parallelism: local queries against the full text)
        h = ops.layernorm_modulate(x, weight=blk.norm2.weight, bias=blk.norm2.bias, eps=cfg.eps)
        a2 = blk.attn2
        q2 = ops.linear(h, a2.to_q.weight, a2.to_q.bias)
        ops.rmsnorm_rope_(q2, a2.norm_q.weight, eps=cfg.eps, head_dim=hd)
        kv = ops.linear(pk.ctx, a2.w_kv, a2.b_kv)
        k2, v2 = kv[:, :D], kv[:, D:]
        ops.rmsnorm_rope_(k2, a2.norm_k.weight, eps=cfg.eps, head_dim=hd)
        L = pk.text_len
        o2 = ops.attention(q2.reshape(pk.batch, pk.seq_local, D), k2.reshape(pk.batch, L, D),
                           v2.reshape(pk.batch, L, D), Hh).reshape(pk.batch * pk.seq_local, D)
        x = ops.linear(o2, a2.to_out[0].weight, a2.to_out[0].bias, residual=x, out=x if x.is_cuda else None)
        # --- feed forward
        h = ops.layernorm_modulate(x, scale=m[:, 4], shift=m[:, 3], eps=cfg.eps, rows_per_batch=rpb)
        f = ops.linear(h, blk.ffn.net[0].proj.weight, blk.ffn.net[0].proj.bias, act="gelu")
        x = ops.linear(f, blk.ffn.net[2].weight, blk.ffn.net[2].bias, residual=x, gate=m[:, 5], rows_per_batch=rpb,
                       out=x if x.is_cuda else None)
        pk.x = x
        pk.next_block = i + 1
        return pk

    def predict(self, pk: WanPacket, pctx=None) -> torch.Tensor:
        """norm_out + proj_out (+ sequence all-gather) + unpatchify -> [B, C, F, H, W] (model dtype)."""
        pctx = pctx or LocalAttention()
        cfg = self.cfg
        per_tok = pk.temb.shape[0] != pk.batch
        rpb = 1 if per_tok else pk.seq_local
        m = self.scale_shift_table.float() + pk.temb[:, None, :]
        h = ops.layernorm_modulate(pk.x, scale=m[:, 1], shift=m[:, 0], eps=cfg.eps, rows_per_batch=rpb)
        y = ops.linear(h, self.proj_out.weight, self.proj_out.bias)
        y = pctx.gather_sequence(y, pk.batch, pk.seq_local)
        return self.unpatchify(y, pk.grid, pk.batch)

    def forward(self, latents, timestep, context, pctx=None):
        pk = self.begin(latents, timestep, context, pctx)
        for i in range(self.cfg.layers):
            self.forward_block(i, pk, pctx)
        return self.predict(pk, pctx)
