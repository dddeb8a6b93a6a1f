"""Flash attention on tcgen05/TMEM (self, cross and packed-varlen).

Inputs are token-major bf16 views ``[tokens, heads * head_dim]`` (or
``[B, S, heads * head_dim]``); q/k/v may be column slices of one fused QKV
buffer (any row stride).  ``cu_seqlens_q/k`` select the packed-varlen mode used
by SD3.5 continuous batching (reference: workers/ditserve/models/sd35_batch.py:19-117).
"""
from __future__ import annotations

import math

import torch

from ._ext import kernel, status_word, use_kernels


def attention_reference(q, k, v, heads, heads_kv=None, cu_seqlens_q=None, cu_seqlens_k=None, scale=None,
                        return_lse=False):
    """fp32 PyTorch statement of the kernel (CPU path and test oracle)."""
    heads_kv = heads_kv or heads
    width = q.shape[-1]
    d = width // heads
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    if cu_seqlens_q is None:
        if q.dim() == 2:
            q, k, v = q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0)
            squeeze = True
        else:
            squeeze = False
        B, Sq, _ = q.shape
        Sk = k.shape[1]
        qh = q.float().reshape(B, Sq, heads, d).transpose(1, 2)
        kh = k.float().reshape(B, Sk, heads_kv, d).transpose(1, 2)
        vh = v.float().reshape(B, Sk, heads_kv, d).transpose(1, 2)
        if heads_kv != heads:
            kh = kh.repeat_interleave(heads // heads_kv, dim=1)
            vh = vh.repeat_interleave(heads // heads_kv, dim=1)
        s = (qh @ kh.transpose(-1, -2)) * scale
        lse = torch.logsumexp(s, dim=-1)
        o = (torch.softmax(s, dim=-1) @ vh).transpose(1, 2).reshape(B, Sq, heads * d).to(q.dtype)
        if squeeze:
            o, lse = o[0], lse[0]
        return (o, lse) if return_lse else o
    outs, lses = [], []
    cq = cu_seqlens_q.tolist()
    ck = cu_seqlens_k.tolist()
    for i in range(len(cq) - 1):
        o, l = attention_reference(q[cq[i]:cq[i + 1]], k[ck[i]:ck[i + 1]], v[ck[i]:ck[i + 1]], heads, heads_kv,
                                   scale=scale, return_lse=True)
        outs.append(o)
        lses.append(l)
    o = torch.cat(outs, 0)
    return (o, torch.cat(lses, -1)) if return_lse else o


def segments_reference(q, k, v, heads, seg_table, scale=None, heads_kv=None):
    """Dual-range segments: rows [qa0,qa1) u [qb0,qb1) attend to [ka0,ka1) u [kb0,kb1)."""
    out = torch.zeros(q.shape[0], q.shape[1], dtype=q.dtype)
    for row in seg_table.tolist():
        qa0, qa1, qb0, qb1, ka0, ka1, kb0, kb1 = row
        qi = torch.cat([torch.arange(qa0, qa1), torch.arange(qb0, qb1)])
        ki = torch.cat([torch.arange(ka0, ka1), torch.arange(kb0, kb1)])
        if len(qi) == 0 or len(ki) == 0:
            continue
        o = attention_reference(q[qi], k[ki], v[ki], heads, heads_kv, scale=scale)
        out[qi] = o.to(out.dtype)
    return out


def segment_table(segments) -> torch.Tensor:
    """[(qa0, qa1, qb0, qb1, ka0, ka1, kb0, kb1), ...] -> int32 [n, 8]."""
    return torch.tensor([list(s) for s in segments], dtype=torch.int32)


def attention_segments(q, k, v, heads, seg_table: torch.Tensor, *, scale=None, out=None, heads_kv=None):
    """Attention over dual-range segments of one packed buffer (MMDiT joint attention)."""
    heads_kv = heads_kv or heads
    if not use_kernels(q, k, v):
        o = segments_reference(q, k, v, heads, seg_table, scale, heads_kv)
        if out is not None:
            rows = torch.zeros(q.shape[0], dtype=torch.bool)
            for r in seg_table.tolist():
                rows[r[0]:r[1]] = True
                rows[r[2]:r[3]] = True
            out[rows] = o[rows]
            return out
        return o
    d = q.shape[-1] // heads
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    tbl = seg_table.to(torch.int32)
    cpu = tbl.cpu()
    blocks = int(((cpu[:, 1] - cpu[:, 0] + 255) // 256 + (cpu[:, 3] - cpu[:, 2] + 255) // 256).max().item())
    if out is None:
        out = torch.empty(q.shape[0], q.shape[1], device=q.device, dtype=torch.bfloat16)
    kernel("attention")(q, k, v, out, None, tbl.shape[0], 0, 0, None, None, 0, heads, heads_kv, d, float(scale),
                        status_word(q.device), tbl.to(q.device).contiguous(), blocks, [], [])
    return out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, *, heads_kv: int | None = None,
              cu_seqlens_q: torch.Tensor | None = None, cu_seqlens_k: torch.Tensor | None = None,
              max_seqlen_q: int | None = None, scale: float | None = None, out: torch.Tensor | None = None,
              return_lse: bool = False, kv_extra: list | None = None):
    """``kv_extra`` = [(k_i, v_i), ...]: extra key/value sources laid out like k/v (ring chunks);
    every query attends to the keys of all sources."""
    heads_kv = heads_kv or heads
    if not use_kernels(q, k, v):
        if kv_extra:
            cat = 1 if k.dim() == 3 else 0
            k = torch.cat([k] + [e[0] for e in kv_extra], cat)
            v = torch.cat([v] + [e[1] for e in kv_extra], cat)
        return attention_reference(q, k, v, heads, heads_kv, cu_seqlens_q, cu_seqlens_k, scale, return_lse)
    width = q.shape[-1]
    d = width // heads
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    if q.dim() == 3:
        B, Sq, _ = q.shape
        Sk = k.shape[1]
        q2, k2, v2 = q.reshape(B * Sq, width), k.reshape(B * Sk, -1), v.reshape(B * Sk, -1)
    else:
        q2, k2, v2 = q, k, v
        if cu_seqlens_q is None:
            B, Sq, Sk = 1, q.shape[0], k.shape[0]
        else:
            B, Sq, Sk = cu_seqlens_q.numel() - 1, 0, 0
    if out is None:
        out = torch.empty(q2.shape[0], width, device=q.device, dtype=torch.bfloat16)
    o2 = out.reshape(q2.shape[0], width)
    lse = torch.empty(heads, q2.shape[0], device=q.device, dtype=torch.float32) if return_lse else None
    cq = cu_seqlens_q.to(torch.int32) if cu_seqlens_q is not None else None
    ckk = cu_seqlens_k.to(torch.int32) if cu_seqlens_k is not None else None
    if cq is not None and max_seqlen_q is None:
        max_seqlen_q = int((cq[1:] - cq[:-1]).max().item())
    ke = [e[0].reshape(k2.shape) for e in (kv_extra or [])]
    ve = [e[1].reshape(v2.shape) for e in (kv_extra or [])]
    kernel("attention")(q2, k2, v2, o2, lse, B, Sq, Sk, cq, ckk, int(max_seqlen_q or 0), heads, heads_kv, d,
                        float(scale), status_word(q.device), None, 0, ke, ve)
    o = out.reshape(*q.shape[:-1], width)
    return (o, lse) if return_lse else o
