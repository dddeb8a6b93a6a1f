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
                        return_lse=False, mask=None):
    """fp32 PyTorch statement of the kernel (CPU path and test oracle); ``mask``: optional bool
    [seq_q, seq_k] of the (query, key) pairs that may attend (uniform batches only)."""
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
        if mask is not None:
            s = s.masked_fill(~mask.to(s.device), float("-inf"))
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
                        status_word(q.device), tbl.to(q.device).contiguous(), blocks, [], [], None, None)
    return out


# ---------------------------------------------------------------------------------------------
# Block-sparse attention: a boolean [query blocks, key tiles] mask at the kernel's granularity
# (a CTA's 256 query rows x a 128-key tile) names the key tiles each query block attends to;
# the kernel streams only those tiles (one online softmax over them).  Sliding-window and
# 3-D tile-window patterns for video tokens are built by the helpers below.  Reference: the
# sparse attention masks of the reference's engine (SSTA / sliding-tile attention,
# workers/xfuser/.../ssta.py), rebuilt at this kernel's tile granularity.
SPARSE_Q_BLOCK = 256
SPARSE_K_BLOCK = 128


def block_sparse_table(block_mask: torch.Tensor, device=None):
    """bool [nq, nk] -> (offsets int32 [nq + 1], index int32 [nnz]) on ``device``."""
    m = torch.as_tensor(block_mask, dtype=torch.bool).cpu()
    if m.dim() != 2:
        raise ValueError("block_mask must be [query blocks, key tiles]")
    counts = m.sum(1)
    if bool((counts == 0).any()):
        raise ValueError("every query block must attend to at least one key tile")
    offsets = torch.zeros(m.shape[0] + 1, dtype=torch.int32)
    offsets[1:] = torch.cumsum(counts, 0).to(torch.int32)
    index = m.nonzero()[:, 1].to(torch.int32)
    return offsets.to(device).contiguous(), index.to(device).contiguous()


def token_mask(block_mask: torch.Tensor, seq_q: int, seq_k: int) -> torch.Tensor:
    """The [seq_q, seq_k] token mask that a block mask stands for."""
    m = torch.as_tensor(block_mask, dtype=torch.bool).cpu()
    qi = torch.arange(seq_q) // SPARSE_Q_BLOCK
    ki = torch.arange(seq_k) // SPARSE_K_BLOCK
    return m[qi][:, ki]


def sliding_window_block_mask(seq_q: int, seq_k: int, window: int) -> torch.Tensor:
    """Key tiles holding any key within ``window`` positions of any query of the block."""
    nq = -(-seq_q // SPARSE_Q_BLOCK)
    nk = -(-seq_k // SPARSE_K_BLOCK)
    q0 = torch.arange(nq) * SPARSE_Q_BLOCK
    q1 = torch.clamp(q0 + SPARSE_Q_BLOCK, max=seq_q) - 1
    k0 = torch.arange(nk) * SPARSE_K_BLOCK
    k1 = torch.clamp(k0 + SPARSE_K_BLOCK, max=seq_k) - 1
    # intervals [q0 - w, q1 + w] and [k0, k1] overlap
    return (k0[None, :] <= q1[:, None] + window) & (k1[None, :] >= q0[:, None] - window)


def tile_window_block_mask(grid, window) -> torch.Tensor:
    """Video tokens in (t, h, w) raster order; a query attends to keys whose (t, h, w) lie
    within ``window`` = (wt, wh, ww) of its own in every axis.  Returns the block mask that
    covers every such pair (a block pair is kept when any of its token pairs is in range)."""
    T, H, W = grid
    wt, wh, ww = window
    n = T * H * W
    idx = torch.arange(n)
    t, h, w = idx // (H * W), (idx // W) % H, idx % W
    nq = -(-n // SPARSE_Q_BLOCK)
    nk = -(-n // SPARSE_K_BLOCK)

    def boxes(size):
        nb = -(-n // size)
        lo, hi = [], []
        for b in range(nb):
            sl = slice(b * size, min(n, (b + 1) * size))
            c = torch.stack([t[sl], h[sl], w[sl]], 1)
            lo.append(c.min(0).values)
            hi.append(c.max(0).values)
        return torch.stack(lo), torch.stack(hi)
    qlo, qhi = boxes(SPARSE_Q_BLOCK)
    klo, khi = boxes(SPARSE_K_BLOCK)
    win = torch.tensor([wt, wh, ww])
    # bounding boxes within the window in every axis (a cover of the token-level pattern)
    ok = (klo[None, :, :] <= qhi[:, None, :] + win) & (khi[None, :, :] >= qlo[:, None, :] - win)
    assert ok.shape[:2] == (nq, nk)
    return ok.all(-1)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, *, heads_kv: int | None = None,
              cu_seqlens_q: torch.Tensor | None = None, cu_seqlens_k: torch.Tensor | None = None,
              max_seqlen_q: int | None = None, scale: float | None = None, out: torch.Tensor | None = None,
              return_lse: bool = False, kv_extra: list | None = None, block_mask: torch.Tensor | None = None,
              block_table=None):
    """``kv_extra`` = [(k_i, v_i), ...]: extra key/value sources laid out like k/v (ring chunks);
    every query attends to the keys of all sources.  ``block_mask``: bool [query blocks of
    256 rows, key tiles of 128] for block-sparse attention (uniform batches, one KV source);
    ``block_table``: the same as a prebuilt ``block_sparse_table`` on the device."""
    heads_kv = heads_kv or heads
    sparse = block_mask is not None or block_table is not None
    if sparse and (cu_seqlens_q is not None or kv_extra):
        raise ValueError("block-sparse attention takes uniform batches and one KV source")
    if not use_kernels(q, k, v):
        if sparse:
            if block_mask is None:
                raise ValueError("the CPU path needs block_mask")
            Sq, Sk = q.shape[-2], k.shape[-2]
            return attention_reference(q, k, v, heads, heads_kv, scale=scale, return_lse=return_lse,
                                       mask=token_mask(block_mask, Sq, Sk))
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
    boff = bidx = None
    if sparse:
        if block_table is None:
            nq, nk = -(-Sq // SPARSE_Q_BLOCK), -(-Sk // SPARSE_K_BLOCK)
            if tuple(block_mask.shape) != (nq, nk):
                raise ValueError(f"block_mask must be [{nq}, {nk}] for {Sq} queries and {Sk} keys")
            block_table = block_sparse_table(block_mask, q.device)
        boff, bidx = block_table
    kernel("attention")(q2, k2, v2, o2, lse, B, Sq, Sk, cq, ckk, int(max_seqlen_q or 0), heads, heads_kv, d,
                        float(scale), status_word(q.device), None, 0, ke, ve, boff, bidx)
    o = out.reshape(*q.shape[:-1], width)
    return (o, lse) if return_lse else o
