"""Fused LayerNorm/adaLN modulation and RMS qk-norm + rotary embedding.

Reference semantics: diffusers WanTransformerBlock as driven by
workers/ditserve/models/wan/block.py:282-297 (``norm(h.float()) * (1 + scale) + shift``)
and the Wan attention processor's RMS qk-norm across heads followed by the
interleaved-pair RoPE (workers/xfuser/model_executor/models/transformers/transformer_wan.py:158-191).
"""
from __future__ import annotations

import torch

from ._ext import kernel, use_kernels


def _batch_rows(x2, rows_per_batch, mod, row_batch=None):
    if mod is None:
        return None
    m = mod.float()
    if m.dim() == 1:
        m = m.unsqueeze(0)
    if row_batch is not None:
        return m[row_batch.long().to(m.device)]
    rpb = rows_per_batch or x2.shape[0]
    return m.repeat_interleave(rpb, dim=0)[: x2.shape[0]]


def layernorm_modulate_reference(x, scale=None, shift=None, weight=None, bias=None, eps=1e-6, rows_per_batch=None,
                                 row_batch=None):
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).float()
    y = torch.nn.functional.layer_norm(x2, (x2.shape[-1],), eps=eps)
    if weight is not None:
        y = y * weight.float()
    if bias is not None:
        y = y + bias.float()
    sc = _batch_rows(x2, rows_per_batch, scale, row_batch)
    sh = _batch_rows(x2, rows_per_batch, shift, row_batch)
    if sc is not None:
        y = y * (1 + sc)
    if sh is not None:
        y = y + sh
    return y.to(x.dtype).reshape(shape)


def layernorm_modulate(x: torch.Tensor, scale: torch.Tensor | None = None, shift: torch.Tensor | None = None,
                       weight: torch.Tensor | None = None, bias: torch.Tensor | None = None, eps: float = 1e-6,
                       rows_per_batch: int | None = None, out: torch.Tensor | None = None,
                       row_batch: torch.Tensor | None = None) -> torch.Tensor:
    """y = LN(x) [* w + b] [* (1 + scale[b]) + shift[b]]; scale/shift fp32 [B, D]; the batch index of a
    row is row // rows_per_batch, or row_batch[row] for packed ragged batches."""
    if not use_kernels(x):
        y = layernorm_modulate_reference(x, scale, shift, weight, bias, eps, rows_per_batch, row_batch)
        if out is not None:
            out.copy_(y.reshape(out.shape))
            return out
        return y
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    y = out if out is not None else torch.empty_like(x2)
    y2 = y.reshape(x2.shape)

    def prep(m):
        if m is None:
            return None
        return m.unsqueeze(0) if m.dim() == 1 else m

    sc, sh = prep(scale), prep(shift)
    mod_stride = 0
    if sc is not None:
        mod_stride = sc.stride(0) if sc.shape[0] > 1 else 0
        if sh is not None:
            assert sh.stride(0) == sc.stride(0) or sh.shape[0] == 1, "scale/shift must share a row stride"
    elif sh is not None:
        mod_stride = sh.stride(0) if sh.shape[0] > 1 else 0
    kernel("layernorm_modulate")(x2, y2, sc, sh, mod_stride, int(rows_per_batch or x2.shape[0]), weight, bias,
                                 float(eps), row_batch)
    return y2.reshape(shape)


def rms_norm_reference(x, weight=None, eps=1e-6, groups=1):
    shape = x.shape
    xf = x.float().reshape(*shape[:-1], groups, shape[-1] // groups)
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = y.reshape(shape)
    if weight is not None:
        w = weight.float()
        if groups > 1 and w.numel() == shape[-1] // groups:
            w = w.repeat(groups)
        y = y * w
    return y.to(x.dtype)


def rope_reference(x, cos, sin, head_dim, rows_per_batch=None):
    """Interleaved-pair rotation; cos/sin fp32 [positions, head_dim/2]."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).float()
    M = x2.shape[0]
    rpb = rows_per_batch or M
    pos = torch.arange(M, device=x.device) % rpb
    c = cos[pos].repeat(1, shape[-1] // head_dim)
    s = sin[pos].repeat(1, shape[-1] // head_dim)
    x0, x1 = x2[:, 0::2], x2[:, 1::2]
    y = torch.empty_like(x2)
    y[:, 0::2] = x0 * c - x1 * s
    y[:, 1::2] = x0 * s + x1 * c
    return y.to(x.dtype).reshape(shape)


def rmsnorm_rope_(x: torch.Tensor, weight: torch.Tensor | None, *, groups: int = 1, eps: float = 1e-6,
                  cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
                  rows_per_batch: int | None = None, head_dim: int = 128) -> torch.Tensor:
    """In place: x = rope(rms_norm(x) * w).  ``groups`` = 1 normalises across all
    heads of a token (Wan), ``groups`` = heads normalises each head (SD3.5)."""
    if not use_kernels(x):
        y = rms_norm_reference(x, weight, eps, groups)
        if cos is not None:
            y = rope_reference(y, cos, sin, head_dim, rows_per_batch)
        x.copy_(y)
        return x
    x2 = x if x.dim() == 2 else x.reshape(-1, x.shape[-1])
    width = x2.shape[1] // groups
    kernel("rmsnorm_rope")(x2, weight, width, groups, float(eps), cos, sin, int(rows_per_batch or x2.shape[0]),
                           head_dim, None, 0)
    return x


def rmsnorm_rope_qk_(qkv: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, *, eps: float = 1e-6,
                     cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
                     rows_per_batch: int | None = None, head_dim: int = 128) -> torch.Tensor:
    """In place on the q and k columns of a fused [rows, >= 3D] QKV buffer, in one launch:
    q = rope(rms_norm(q) * wq), k = rope(rms_norm(k) * wk), norms across all heads (Wan)."""
    d = wq.numel()
    q, k = qkv[:, :d], qkv[:, d:2 * d]
    if not use_kernels(qkv):
        rmsnorm_rope_(q, wq, eps=eps, cos=cos, sin=sin, rows_per_batch=rows_per_batch, head_dim=head_dim)
        rmsnorm_rope_(k, wk, eps=eps, cos=cos, sin=sin, rows_per_batch=rows_per_batch, head_dim=head_dim)
        return qkv
    kernel("rmsnorm_rope")(q, wq, d, 1, float(eps), cos, sin, int(rows_per_batch or qkv.shape[0]), head_dim, wk, d)
    return qkv
