"""Implicit-GEMM channels-last convolution (tcgen05) against the fp32 torch statement:
causal 3x3x3 and 2-D 3x3 kernels, 1x1 kernels, every output-tile width the decoder uses,
spatial tails of the 32 x 4 pixel tiles, a ragged RGB output, the residual epilogue and the
halo mode (pad_h = 0: the input carries its own neighbour rows)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from ditserve_b200 import ops


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


CASES = [
    # c_in, c_out, kernel, pad, T_in, H, W
    (96, 96, (3, 3, 3), (1, 1), 3, 10, 40),
    (192, 384, (3, 3, 3), (1, 1), 4, 9, 33),
    (384, 192, (1, 3, 3), (1, 1), 2, 7, 65),
    (32, 3, (3, 3, 3), (1, 1), 3, 12, 36),
    (96, 96, (1, 1, 1), (0, 0), 1, 5, 104),
    (384, 384, (3, 1, 1), (0, 0), 3, 6, 20),
    (96, 64, (3, 3, 3), (0, 1), 3, 12, 40),
]


@pytest.mark.parametrize("c_in,c_out,ks,pad,T,H,W", CASES)
@pytest.mark.parametrize("res", [False, True])
def test_conv_matches_fp32_statement(c_in, c_out, ks, pad, T, H, W, res):
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(c_in + c_out + H)
    w = torch.randn(c_out, c_in, *ks, generator=g) / (c_in * ks[0] * ks[1] * ks[2]) ** 0.5
    b = torch.randn(c_out, generator=g)
    x = torch.randn(T, H, W, c_in, generator=g).bfloat16()
    w2d = ops.conv_weight_2d(w)
    bias = ops.conv_bias(b, w2d.shape[0])
    shape = (T - ks[0] + 1, H + 2 * pad[0] - ks[1] + 1, W + 2 * pad[1] - ks[2] + 1, c_out)
    r = torch.randn(shape, generator=g).bfloat16() if res else None
    y = ops.conv_cl(x.to(dev), w2d.to(dev), bias.to(dev), ks, pad, c_out, residual=None if r is None else r.to(dev))
    ops.check_status(dev)
    ref = ops.conv_cl_reference(x.float(), w2d.float(), bias.float(), ks, pad, c_out,
                                residual=None if r is None else r.float())
    assert y.shape == ref.shape
    assert _rel(y, ref) < 1e-2, _rel(y, ref)


def test_conv_output_guard_band():
    """A conv writing into the interior of a larger buffer leaves the sentinel rows around it
    untouched (the halo layout writes outputs between neighbour rows)."""
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(3, 10, 40, 96, generator=g).bfloat16().to(dev)
    w2d = ops.conv_weight_2d(torch.randn(96, 96, 3, 3, 3, generator=g) / 50).to(dev)
    buf = torch.full((1, 12, 40, 96), 1024.0, device=dev, dtype=torch.bfloat16)
    ops.conv_cl(x, w2d, None, (3, 3, 3), (1, 1), 96, out=buf[:, 1:11])
    torch.cuda.synchronize()
    ops.check_status(dev)
    assert torch.all(buf[:, 0] == 1024.0) and torch.all(buf[:, 11] == 1024.0)
