"""DPM-Solver++ multistep (data prediction) over a flow-matching velocity model.

Lu et al., "DPM-Solver++: Fast Solver for Guided Sampling of Diffusion Probabilistic
Models" (2022), Alg. 2 (multistep second order) and the third-order multistep
extension of the DPM-Solver paper (Lu et al., 2022, Sec. 3.3).  For a flow sample
x_s = (1 - s) x_0 + s eps the noise schedule is alpha_s = 1 - s, sigma_s = s and the
half log-SNR is lambda(s) = log(1 - s) - log(s).  The DiT predicts the velocity v and
the data estimate is m = x - s v.  One step from s0 to t, h = lambda(t) - lambda(s0),
phi = expm1(-h), with the previous estimates m1 (at s1) and m2 (at s2):

    order 1:  x_t = (t/s0) x - (1-t) phi m0
    order 2:  r0 = (lambda(s0) - lambda(s1)) / h,  D1 = (m0 - m1) / r0
              midpoint:  x_t = (t/s0) x - (1-t) phi m0 - (1-t) phi D1 / 2
              heun:      x_t = (t/s0) x - (1-t) phi m0 + (1-t) (phi/h + 1) D1
    order 3:  r1 = (lambda(s1) - lambda(s2)) / h,
              D1_0 = (m0 - m1)/r0,  D1_1 = (m1 - m2)/r1,
              D1 = D1_0 + r0/(r0+r1) (D1_0 - D1_1),  D2 = (D1_0 - D1_1)/(r0+r1)
              x_t = (t/s0) x - (1-t) phi m0 + (1-t)(phi/h + 1) D1 - (1-t)((phi+h)/h^2 - 1/2) D2

Every form is linear in x, the current estimate and the stored ones, so a step is one
launch of the fused ``ops.sched_step`` kernel (CFG combine + update + the new estimate
written to the history slab) with host-computed coefficients — the same kernel, and the
same peer-memory CFG variant, as UniPC and Euler.  A step that lands on sigma 0 is first
order (the update reduces to x_t = m0).  Reference: the DPM-Solver multistep scheduler the
reference wraps for patch-parallel stepping
(workers/xfuser/model_executor/schedulers/scheduling_dpmsolver_multistep.py:16-201).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from .. import ops
from .unipc import unipc_flow_sigmas


def _lam(s: float) -> float:
    # the grid's ends (pure data, pure noise) have infinite log-SNR; the update coefficients
    # take their finite limits there
    if s <= 0.0:
        return math.inf
    if s >= 1.0:
        return -math.inf
    return math.log(1.0 - s) - math.log(s)


class DPMSolverFlowScheduler:
    """Stateful DPM-Solver++(1/2/3M); device buffers hold the data-estimate history."""

    KIND = "dpmpp_flow.v1"

    def __init__(self, steps: int, flow_shift: float = 3.0, order: int = 2, solver_type: str = "midpoint",
                 lower_order_final: bool = True, train_steps: int = 1000, sigmas: list[float] | None = None):
        if order not in (1, 2, 3):
            raise ValueError("DPM-Solver++ order must be 1, 2 or 3")
        if solver_type not in ("midpoint", "heun"):
            raise ValueError("solver_type must be midpoint or heun")
        self.steps = int(steps)
        self.flow_shift = float(flow_shift)
        self.order = int(order)
        self.solver_type = solver_type
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
        self.hist_sigmas: list[float] = []   # sigma of each stored estimate, oldest first
        self.hist: list[torch.Tensor] = []    # data estimates, oldest first
        self._spare: list[torch.Tensor] = []

    def timestep(self) -> float:
        return self.timesteps[self.step_index]

    @property
    def done(self) -> bool:
        return self.step_index >= self.steps

    def _alloc(self, like: torch.Tensor) -> torch.Tensor:
        if self._spare:
            return self._spare.pop()
        return torch.empty_like(like, dtype=torch.float32)

    def this_order(self) -> int:
        k = self.step_index
        order = min(self.order, self.lower_order_nums + 1)
        if self.lower_order_final and self.steps < 15:
            order = min(order, self.steps - k)
        if self.sigmas[k + 1] <= 0.0:
            order = 1
        return max(order, 1)

    def coefficients(self) -> tuple[float, dict]:
        """(sigma of this step, predictor coefficients) for ``ops.sched_step``."""
        k = self.step_index
        s0, t = self.sigmas[k], self.sigmas[k + 1]
        order = self.this_order()
        h = _lam(t) - _lam(s0)
        alpha_t = 1.0 - t
        phi = math.expm1(-h)
        # coefficients of (m0, m1, m2)
        m = np.zeros(3, dtype=np.float64)
        m[0] = -alpha_t * phi
        if order >= 2:
            r0 = (_lam(s0) - _lam(self.hist_sigmas[-1])) / h
            d1_0 = np.array([1.0 / r0, -1.0 / r0, 0.0])
            if order == 2:
                if self.solver_type == "midpoint":
                    m += -0.5 * alpha_t * phi * d1_0
                else:
                    m += alpha_t * (phi / h + 1.0) * d1_0
            else:
                r1 = (_lam(self.hist_sigmas[-1]) - _lam(self.hist_sigmas[-2])) / h
                d1_1 = np.array([0.0, 1.0 / r1, -1.0 / r1])
                diff = d1_0 - d1_1
                d1 = d1_0 + r0 / (r0 + r1) * diff
                d2 = diff / (r0 + r1)
                m += alpha_t * (phi / h + 1.0) * d1
                m += -alpha_t * ((phi + h) / (h * h) - 0.5) * d2
        pred = dict(x=t / s0, x0=float(m[0]), hist_coef=[float(m[i]) for i in range(1, order)], order=order)
        return s0, pred

    def step(self, sample: torch.Tensor, cond: torch.Tensor, uncond: torch.Tensor | None = None,
             guidance: float = 1.0, kernel=None) -> torch.Tensor:
        """Advance ``sample`` (fp32, in place) by one step from the model's velocity."""
        if self.done:
            raise RuntimeError("scheduler already finished")
        s0, pred = self.coefficients()
        x0_new = self._alloc(sample)
        pred_args = dict(x=pred["x"], x0=pred["x0"],
                         hist=[self.hist[-(i + 1)] for i in range(pred["order"] - 1)],
                         hist_coef=pred["hist_coef"])
        (kernel or ops.sched_step)(cond, uncond, guidance, sample, s0, None, pred_args, x0_out=x0_new,
                                   last_out=None)
        self.hist.append(x0_new)
        self.hist_sigmas.append(s0)
        while len(self.hist) > max(self.order - 1, 1):
            self._spare.append(self.hist.pop(0))
            self.hist_sigmas.pop(0)
        self.lower_order_nums = min(self.lower_order_nums + 1, self.order)
        self.step_index += 1
        return sample

    def state_dict(self, device: str | torch.device | None = "cpu") -> dict:
        mv = (lambda t: t.detach().to(device, copy=True)) if device is not None else (lambda t: t)
        return dict(kind=self.KIND, steps=self.steps, flow_shift=self.flow_shift, order=self.order,
                    solver_type=self.solver_type, lower_order_final=self.lower_order_final,
                    train_steps=self.train_steps, sigmas=self.custom_sigmas, step_index=self.step_index,
                    lower_order_nums=self.lower_order_nums, hist_sigmas=list(self.hist_sigmas),
                    hist=[mv(t) for t in self.hist])

    @classmethod
    def from_state_dict(cls, sd: dict, device: str | torch.device | None = None) -> "DPMSolverFlowScheduler":
        if sd.get("kind") != cls.KIND:
            raise ValueError("not a DPM-Solver++ flow scheduler state")
        s = cls(sd["steps"], sd["flow_shift"], sd["order"], sd["solver_type"], sd["lower_order_final"],
                sd["train_steps"], sd.get("sigmas"))
        mv = (lambda t: t.to(device, copy=True)) if device is not None else (lambda t: t.clone())
        s.step_index = int(sd["step_index"])
        s.lower_order_nums = int(sd["lower_order_nums"])
        s.hist_sigmas = [float(v) for v in sd["hist_sigmas"]]
        s.hist = [mv(t) for t in sd["hist"]]
        return s
