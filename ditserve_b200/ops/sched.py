"""Fused CFG combine + latent update (one pass over the latent).

The host scheduler (``ditserve_b200.schedulers``) turns one UniPC bh2
predictor/corrector step or one flow-matching Euler step into the linear
coefficients below; this op applies them.  Reference: the CFG combine and
``scheduler.step`` of workers/ditserve/models/wan/block.py:472-486 and
workers/ditserve/models/sd35.py:943-952.
"""
from __future__ import annotations

import torch

from ._ext import kernel, use_kernels


def sched_step_reference(cond, uncond, guidance, sample, sigma, corrector, predictor, x0_out=None, last_out=None):
    v = cond.float() if uncond is None else uncond.float() + guidance * (cond.float() - uncond.float())
    v = v.reshape(sample.shape)
    x = sample.float()
    x0 = x - sigma * v
    xc = x
    if corrector is not None:
        xc = corrector["last_coef"] * corrector["last"].float() + corrector["x0_coef"] * x0
        for buf, coef in zip(corrector.get("hist", []), corrector.get("hist_coef", [])):
            xc = xc + coef * buf.float()
    nx = predictor.get("x", 1.0) * xc + predictor.get("x0", 0.0) * x0 + predictor.get("v", 0.0) * v
    for buf, coef in zip(predictor.get("hist", []), predictor.get("hist_coef", [])):
        nx = nx + coef * buf.float()
    if x0_out is not None:
        x0_out.copy_(x0)
    if last_out is not None:
        last_out.copy_(xc)
    sample.copy_(nx)
    return sample


def sched_step(cond: torch.Tensor, uncond: torch.Tensor | None, guidance: float, sample: torch.Tensor,
               sigma: float, corrector: dict | None, predictor: dict, x0_out: torch.Tensor | None = None,
               last_out: torch.Tensor | None = None) -> torch.Tensor:
    """Update ``sample`` (fp32, in place).  ``corrector``/``predictor`` hold the
    coefficients and history buffers produced by the scheduler."""
    if not use_kernels(sample):
        return sched_step_reference(cond, uncond, guidance, sample, sigma, corrector, predictor, x0_out, last_out)
    c = corrector or {}
    kernel("sched_step")(
        cond.contiguous(), None if uncond is None else uncond.contiguous(), float(guidance), sample, float(sigma),
        corrector is not None, c.get("last"), float(c.get("last_coef", 0.0)), float(c.get("x0_coef", 0.0)),
        list(c.get("hist", [])), [float(v) for v in c.get("hist_coef", [])],
        float(predictor.get("x", 1.0)), float(predictor.get("x0", 0.0)), float(predictor.get("v", 0.0)),
        list(predictor.get("hist", [])), [float(v) for v in predictor.get("hist_coef", [])],
        x0_out, last_out)
    return sample
