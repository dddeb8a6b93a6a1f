"""Linear layers on the tcgen05 GEMM with fused epilogues.

``linear(x, w, b, act=..., residual=..., gate=...)`` computes, in one kernel,

    y = x @ w.T + b                    (act=None)
    y = gelu_tanh(x @ w.T + b)         (act="gelu")
    y = residual + gate * (x @ w.T + b) (gate given; adaLN-Zero gated residual)
    y = residual + (x @ w.T + b)        (residual without gate)

with the weight in nn.Linear layout ``[out, in]``.  The gate is fp32 ``[B, N]``
(any row stride, unit column stride) and row ``m`` of ``x`` belongs to batch
``m // rows_per_batch``.  On CPU the same math runs in fp32 with PyTorch.
Reference call sites: workers/xfuser/model_executor/models/transformers/
transformer_wan.py:50-69 (QKV), :154 (out proj); diffusers FeedForward.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import kernel, status_word, use_kernels

EPI_NONE, EPI_GELU, EPI_GATED_RES, EPI_RES = 0, 1, 2, 3


def gelu_tanh_ref(x: torch.Tensor) -> torch.Tensor:
    return F.gelu(x, approximate="tanh")


def _row_gate(gate, rows, rows_per_batch, row_batch):
    g = gate.float()
    if g.dim() == 1:
        g = g.unsqueeze(0)
    if row_batch is not None:
        return g[row_batch.long().cpu()] if not g.is_cuda else g[row_batch.long()]
    rpb = rows_per_batch or rows
    return g.repeat_interleave(rpb, dim=0)[:rows]


def linear_reference(x, w, b=None, act=None, residual=None, gate=None, rows_per_batch=None, row_batch=None):
    """fp32 PyTorch statement of the fused op (CPU path and test oracle)."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).float()
    y = x2 @ w.float().t()
    if b is not None:
        y = y + b.float()
    if act == "gelu":
        y = gelu_tanh_ref(y)
    if residual is not None:
        r = residual.reshape(-1, y.shape[-1]).float()
        if gate is not None:
            y = r + _row_gate(gate, y.shape[0], rows_per_batch, row_batch) * y
        else:
            y = r + y
    return y.to(x.dtype).reshape(*shape[:-1], w.shape[0])


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None, *, act: str | None = None,
           residual: torch.Tensor | None = None, gate: torch.Tensor | None = None,
           rows_per_batch: int | None = None, out: torch.Tensor | None = None,
           bn: int = 0, row_batch: torch.Tensor | None = None, pair: int = -1) -> torch.Tensor:
    if not use_kernels(x, w):
        y = linear_reference(x, w, b, act, residual, gate, rows_per_batch, row_batch)
        if out is not None:
            out.copy_(y.reshape(out.shape))
            return out
        return y
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M, N = x2.shape[0], w.shape[0]
    if out is None:
        out = torch.empty((M, N), device=x.device, dtype=torch.bfloat16)
    out2 = out.view(M, N) if out.dim() != 2 else out
    epi = EPI_NONE
    r2 = None
    if act == "gelu":
        epi = EPI_GELU
    elif act is not None:
        raise ValueError(f"unsupported activation {act!r}")
    if residual is not None:
        if act is not None:
            raise ValueError("activation and residual epilogues are exclusive")
        r2 = residual.reshape(M, N)
        epi = EPI_GATED_RES if gate is not None else EPI_RES
    gate_stride = 0
    if gate is not None:
        if gate.dim() == 1:
            gate = gate.unsqueeze(0)
        if gate.stride(-1) != 1:
            raise ValueError("gate must have unit column stride")
        gate_stride = gate.stride(0) if gate.shape[0] > 1 else 0
    kernel("gemm")(x2, w, out2, b, epi, r2, gate, gate_stride, int(rows_per_batch or M),
                   status_word(x.device), bn, row_batch, int(pair))
    return out2.reshape(*shape[:-1], N)
