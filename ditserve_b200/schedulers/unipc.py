"""UniPC (bh2, data prediction) over a flow-matching velocity model.

Notation: for a flow sample x_s = (1 - s) x_0 + s eps the "alpha" is 1 - s and
the log-SNR is lambda(s) = log(1 - s) - log(s).  The velocity v predicted by the
DiT gives the data estimate x0 = x - s v.  One step from s0 to t with step
h = lambda(t) - lambda(s0):

predictor UniP-p (p = order):
    x_t = (t/s0) x - (1-t) phi1 m0 - (1-t) B(h) sum_i rho_i D_i
corrector UniC-p (applied at the start of the next step with the new x0):
    x_t = (t/s0) x_prev - (1-t) phi1 m0 - (1-t) B(h) (sum_i rho_i D_i + rho_c (x0_new - m0))

with phi1 = expm1(-h), B(h) = expm1(-h), D_i = (m_i - m0) / r_i and
r_i = (lambda(s_i) - lambda(s0)) / h over the stored data estimates m_i.  The
rho weights solve the small order-conditions system R rho = b with
R[k, i] = r_i^k and b[k] = phi_{k+1}(h) k! / B(h) (UniPC, Alg. 1-2); for a
second-order predictor rho = 1/2.

The sigma grid follows the diffusers flow-sigma recipe used by Wan
(linspace in alpha, shifted by ``flow_shift``, final sigma zero) so that step
counts and shifts mean the same thing as in the reference.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from .. import ops


def unipc_flow_sigmas(steps: int, flow_shift: float = 3.0, train_steps: int = 1000) -> list[float]:
    alphas = np.linspace(1.0, 1.0 / train_steps, steps + 1)
    s = 1.0 - alphas
    s = np.flip(flow_shift * s / (1.0 + (flow_shift - 1.0) * s))[:-1].copy()
    return [float(v) for v in s] + [0.0]


def _lam(s: float) -> float:
    # the grid's ends (pure data, pure noise) have infinite log-SNR; the update coefficients
    # take their finite limits there
    if s <= 0.0:
        return math.inf
    if s >= 1.0:
        return -math.inf
    return math.log(1.0 - s) - math.log(s)


def _rho(rks: list[float], hh: float, bh: float, order: int, predictor: bool) -> list[float]:
    """Solve the UniPC order conditions (rks includes the trailing 1.0)."""
    h_phi_1 = math.expm1(hh)
    h_phi_k = h_phi_1 / hh - 1.0 if math.isfinite(hh) else -1.0
    fact = 1.0
    R, b = [], []
    for i in range(1, order + 1):
        R.append([r ** (i - 1) for r in rks])
        b.append(h_phi_k * fact / bh)
        fact *= i + 1
        h_phi_k = (h_phi_k / hh - 1.0 / fact) if math.isfinite(hh) else -1.0 / fact
    R = np.array(R, dtype=np.float64)
    b = np.array(b, dtype=np.float64)
    if predictor:
        if order == 2:
            return [0.5]
        return list(np.linalg.solve(R[:-1, :-1], b[:-1]))
    if order == 1:
        return [0.5]
    return list(np.linalg.solve(R, b))


class UniPCFlowScheduler:
    """Stateful UniPC solver; device buffers hold the data-estimate history."""

    def __init__(self, steps: int, flow_shift: float = 3.0, order: int = 2, lower_order_final: bool = True,
                 train_steps: int = 1000, sigmas: list[float] | None = None):
        if order not in (1, 2, 3):
            raise ValueError("UniPC order must be 1, 2 or 3")
        self.steps = int(steps)
        self.flow_shift = float(flow_shift)
        self.order = int(order)
        self.lower_order_final = bool(lower_order_final)
        self.train_steps = int(train_steps)
        self.custom_sigmas = None if sigmas is None else [float(v) for v in sigmas]
        if self.custom_sigmas is not None:
            if len(self.custom_sigmas) != self.steps + 1:
                raise ValueError("sigmas must hold steps + 1 values (the last one the terminal sigma)")
            self.sigmas = list(self.custom_sigmas)
        else:
            self.sigmas = unipc_flow_sigmas(self.steps, self.flow_shift, self.train_steps)
        self.timesteps = [s * self.train_steps for s in self.sigmas[:-1]]
        self.step_index = 0
        self.lower_order_nums = 0
        self.this_order = 0
        self.hist_sigmas: list[float] = []   # sigma of each stored x0, oldest first
        self.hist: list[torch.Tensor] = []    # x0 estimates, oldest first
        self.last: torch.Tensor | None = None
        self._spare: list[torch.Tensor] = []

    # ------------------------------------------------------------------
    def timestep(self) -> float:
        return self.timesteps[self.step_index]

    @property
    def done(self) -> bool:
        return self.step_index >= self.steps

    def _alloc(self, like: torch.Tensor) -> torch.Tensor:
        if self._spare:
            return self._spare.pop()
        return torch.empty_like(like, dtype=torch.float32)

    def coefficients(self):
        """Corrector/predictor coefficients of the current step (host floats)."""
        k = self.step_index
        s_cur = self.sigmas[k]
        corr = None
        if k > 0 and self.last is not None:
            c_order = self.this_order
            s0 = self.hist_sigmas[-1]
            t = s_cur
            h = _lam(t) - _lam(s0)
            hh = -h
            alpha_t = 1.0 - t
            phi1 = math.expm1(hh)
            bh = math.expm1(hh)
            rks, dcoef = [], []
            for i in range(1, c_order):
                si = self.hist_sigmas[-(i + 1)]
                rks.append((_lam(si) - _lam(s0)) / h)
            rks.append(1.0)
            rhos = _rho(rks, hh, bh, c_order, predictor=False)
            c_x0 = -alpha_t * bh * rhos[-1]
            c_m0 = -alpha_t * phi1 + alpha_t * bh * rhos[-1]
            hist_coef = []
            for i in range(c_order - 1):
                c_m0 += alpha_t * bh * rhos[i] / rks[i]
                hist_coef.append(-alpha_t * bh * rhos[i] / rks[i])
            corr = dict(last_coef=t / s0, x0_coef=c_x0, m0_coef=c_m0, hist_coef=hist_coef, order=c_order)
        # order of this step's predictor
        this_order = min(self.order, self.steps - k) if self.lower_order_final else self.order
        this_order = min(this_order, self.lower_order_nums + 1)
        s0 = s_cur
        t = self.sigmas[k + 1]
        h = _lam(t) - _lam(s0)
        hh = -h
        alpha_t = 1.0 - t
        phi1 = math.expm1(hh)
        bh = math.expm1(hh)
        pred = dict(x=t / s0, x0=-alpha_t * phi1, hist_coef=[], order=this_order)
        if this_order > 1:
            rks = []
            for i in range(1, this_order):
                si = self.hist_sigmas[-i]
                rks.append((_lam(si) - _lam(s0)) / h)
            rks.append(1.0)
            rhos = _rho(rks, hh, bh, this_order, predictor=True)
            for i in range(this_order - 1):
                pred["x0"] += alpha_t * bh * rhos[i] / rks[i]
                pred["hist_coef"].append(-alpha_t * bh * rhos[i] / rks[i])
        return s_cur, corr, pred

    def step(self, sample: torch.Tensor, cond: torch.Tensor, uncond: torch.Tensor | None = None,
             guidance: float = 1.0, kernel=None) -> torch.Tensor:
        """Advance ``sample`` (fp32, in place) by one step from the model's velocity."""
        if self.done:
            raise RuntimeError("scheduler already finished")
        s_cur, corr, pred = self.coefficients()
        x0_new = self._alloc(sample)
        corr_args = None
        last_out = None
        if corr is not None:
            m = corr["order"]
            hist_bufs = [self.hist[-1]] + [self.hist[-(i + 2)] for i in range(m - 1)]
            corr_args = dict(last=self.last, last_coef=corr["last_coef"], x0_coef=corr["x0_coef"],
                             hist=hist_bufs, hist_coef=[corr["m0_coef"]] + corr["hist_coef"])
            last_out = self.last
        else:
            last_out = self._alloc(sample) if self.last is None else self.last
        pred_args = dict(x=pred["x"], x0=pred["x0"],
                         hist=[self.hist[-(i + 1)] for i in range(pred["order"] - 1)],
                         hist_coef=pred["hist_coef"])
        (kernel or ops.sched_step)(cond, uncond, guidance, sample, s_cur, corr_args, pred_args, x0_out=x0_new,
                                   last_out=last_out)
        self.last = last_out
        self.hist.append(x0_new)
        self.hist_sigmas.append(s_cur)
        while len(self.hist) > self.order:
            self._spare.append(self.hist.pop(0))
            self.hist_sigmas.pop(0)
        self.this_order = pred["order"]
        self.lower_order_nums = min(self.lower_order_nums + 1, self.order)
        self.step_index += 1
        return sample

    # ------------------------------------------------------------------
    def state_dict(self, device: str | torch.device | None = "cpu") -> dict:
        mv = (lambda t: t.detach().to(device, copy=True)) if device is not None else (lambda t: t)
        return dict(kind="unipc_flow.v1", steps=self.steps, flow_shift=self.flow_shift, order=self.order,
                    lower_order_final=self.lower_order_final, train_steps=self.train_steps,
                    sigmas=self.custom_sigmas, step_index=self.step_index, lower_order_nums=self.lower_order_nums,
                    this_order=self.this_order, hist_sigmas=list(self.hist_sigmas),
                    hist=[mv(t) for t in self.hist], last=None if self.last is None else mv(self.last))

    @classmethod
    def from_state_dict(cls, sd: dict, device: str | torch.device | None = None) -> "UniPCFlowScheduler":
        if sd.get("kind") != "unipc_flow.v1":
            raise ValueError("not a UniPC flow scheduler state")
        s = cls(sd["steps"], sd["flow_shift"], sd["order"], sd["lower_order_final"], sd["train_steps"],
                sd.get("sigmas"))
        mv = (lambda t: t.to(device, copy=True)) if device is not None else (lambda t: t.clone())
        s.step_index = int(sd["step_index"])
        s.lower_order_nums = int(sd["lower_order_nums"])
        s.this_order = int(sd["this_order"])
        s.hist_sigmas = [float(v) for v in sd["hist_sigmas"]]
        s.hist = [mv(t) for t in sd["hist"]]
        s.last = None if sd["last"] is None else mv(sd["last"])
        return s
