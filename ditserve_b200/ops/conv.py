"""Channels-last convolution on the implicit-GEMM tcgen05 kernel.

``conv_cl(x, w2d, bias, kernel, pad, c_out)`` computes, for x = [T, H, W, C_in] (channels
last, batch folded away by the caller):

    y[t, h, w, o] = bias[o] + sum_{kt, kh, kw, c} W[o, c, kt, kh, kw] * x[t + kt, h + kh - ph, w + kw - pw, c]

valid in time (T_out = T - KT + 1: causal frames are already in x) and zero-padded by
``pad = (ph, pw)`` in space (ph = 0 when x carries its own halo rows, as under patch
parallelism).  ``residual`` (shaped like y) is added in the epilogue.  ``w2d`` is the weight
in the kernel's layout, built once by ``conv_weight_2d``.  CPU tensors run the same math
through ``torch.nn.functional.conv3d`` in fp32 (the CPU path and the test oracle).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import kernel, status_word, use_kernels


def padded(n: int, multiple: int = 32) -> int:
    return (n + multiple - 1) // multiple * multiple


def conv_weight_2d(weight: torch.Tensor, c_in_pad: int | None = None, c_out_pad: int | None = None) -> torch.Tensor:
    """[C_out, C_in, KT, KH, KW] (or [C_out, C_in, KH, KW]) -> [C_out_pad, KT*KH*KW*C_in_pad] bf16,
    tap-major then input channel, zero-padded channels."""
    w = weight if weight.dim() == 5 else weight.unsqueeze(2)
    c_out, c_in = w.shape[0], w.shape[1]
    c_in_pad = c_in_pad or padded(c_in)
    c_out_pad = c_out_pad or padded(c_out)
    full = torch.zeros((c_out_pad, c_in_pad) + tuple(w.shape[2:]), dtype=w.dtype, device=w.device)
    full[:c_out, :c_in] = w
    return full.permute(0, 2, 3, 4, 1).reshape(c_out_pad, -1).contiguous().to(torch.bfloat16)


def conv_bias(bias: torch.Tensor | None, c_out_pad: int) -> torch.Tensor | None:
    if bias is None:
        return None
    out = torch.zeros(c_out_pad, dtype=torch.bfloat16, device=bias.device)
    out[:bias.numel()] = bias.to(torch.bfloat16)
    return out


def conv_cl_reference(x, w2d, bias, kernel_size, pad, c_out, residual=None):
    """fp32 statement of the kernel's math (CPU path and test oracle)."""
    kt, kh, kw = kernel_size
    c_in = x.shape[-1]
    c_out_pad = w2d.shape[0]
    if w2d.shape[1] != kt * kh * kw * c_in:
        raise ValueError("weight K does not match the kernel size and the input channels")
    w = w2d.float().reshape(c_out_pad, kt, kh, kw, c_in).permute(0, 4, 1, 2, 3)
    xi = x.float().permute(3, 0, 1, 2).unsqueeze(0)  # [1, C, T, H, W]
    y = F.conv3d(F.pad(xi, (pad[1], pad[1], pad[0], pad[0], 0, 0)), w,
                 None if bias is None else bias.float())
    y = y[0].permute(1, 2, 3, 0)[..., :c_out]
    if residual is not None:
        y = y + residual.float()
    return y.to(x.dtype)


def conv_cl(x: torch.Tensor, w2d: torch.Tensor, bias: torch.Tensor | None, kernel_size: tuple, pad: tuple,
            c_out: int, residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
            bn: int = 0) -> torch.Tensor:
    kt, kh, kw = kernel_size
    if not use_kernels(x):
        y = conv_cl_reference(x, w2d, bias, kernel_size, pad, c_out, residual)
        if out is not None:
            out.copy_(y)
            return out
        return y
    T, H, W, _ = x.shape
    shape = (T - kt + 1, H + 2 * pad[0] - kh + 1, W + 2 * pad[1] - kw + 1, c_out)
    if out is None:
        out = torch.empty(shape, device=x.device, dtype=torch.bfloat16)
    kernel("conv")(x.contiguous(), w2d, out, bias, residual, kt, kh, kw, pad[0], pad[1], status_word(x.device), bn)
    return out
