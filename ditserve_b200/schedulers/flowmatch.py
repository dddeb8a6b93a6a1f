"""Flow-matching Euler solver with static or resolution-dependent shift.

Grid (the diffusers FlowMatchEulerDiscrete recipe the reference's SD3.5 path
relies on): a linspace of timesteps between the shifted training sigma range
[shift(1/T), 1], divided by T, then shifted again; a terminal sigma of 0.
Static shift:  s' = k s / (1 + (k - 1) s).
Dynamic shift: s' = e^mu / (e^mu + (1/s - 1)), with mu linear in the image
token count between (base_seq_len, base_shift) and (max_seq_len, max_shift).
Update: x <- x + (s_next - s) v, applied by the fused ``ops.sched_step``.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from .. import ops


def mu_for_seq_len(seq_len: int, base_seq_len: int = 256, max_seq_len: int = 4096, base_shift: float = 0.5,
                   max_shift: float = 1.16) -> float:
    m = (max_shift - base_shift) / (max_seq_len - base_seq_len)
    return seq_len * m + (base_shift - m * base_seq_len)


def _shift(s: np.ndarray, shift: float, mu: float | None) -> np.ndarray:
    if mu is not None:
        return math.exp(mu) / (math.exp(mu) + (1.0 / s - 1.0))
    return shift * s / (1.0 + (shift - 1.0) * s)


def flow_shift_sigmas(steps: int, shift: float = 3.0, mu: float | None = None, train_steps: int = 1000) -> list[float]:
    train = np.linspace(1, train_steps, train_steps)[::-1].copy() / train_steps
    if mu is None:
        train = _shift(train, shift, None)
    s_max, s_min = float(train[0]), float(train[-1])
    t = np.linspace(s_max * train_steps, s_min * train_steps, steps)
    s = _shift(t / train_steps, shift, mu)
    return [float(v) for v in s] + [0.0]


class FlowMatchEulerScheduler:
    def __init__(self, steps: int, shift: float = 3.0, mu: float | None = None, train_steps: int = 1000,
                 sigmas: list[float] | None = None):
        self.steps = int(steps)
        self.shift = float(shift)
        self.mu = None if mu is None else float(mu)
        self.train_steps = int(train_steps)
        # an explicit grid (steps + 1 values) replaces the shifted linspace, e.g. the UniPC grid
        # so that an Euler run of a Wan request walks the same sigmas as its UniPC run
        self.custom_sigmas = None if sigmas is None else [float(v) for v in sigmas]
        if self.custom_sigmas is not None:
            if len(self.custom_sigmas) != self.steps + 1:
                raise ValueError("sigmas must hold steps + 1 values (the last one the terminal sigma)")
            self.sigmas = list(self.custom_sigmas)
        else:
            self.sigmas = flow_shift_sigmas(self.steps, self.shift, self.mu, self.train_steps)
        self.timesteps = [s * self.train_steps for s in self.sigmas[:-1]]
        self.step_index = 0

    def timestep(self) -> float:
        return self.timesteps[self.step_index]

    @property
    def done(self) -> bool:
        return self.step_index >= self.steps

    def step(self, sample: torch.Tensor, cond: torch.Tensor, uncond: torch.Tensor | None = None,
             guidance: float = 1.0, kernel=None) -> torch.Tensor:
        if self.done:
            raise RuntimeError("scheduler already finished")
        s, s_next = self.sigmas[self.step_index], self.sigmas[self.step_index + 1]
        (kernel or ops.sched_step)(cond, uncond, guidance, sample, s, None, dict(x=1.0, x0=0.0, v=s_next - s))
        self.step_index += 1
        return sample

    def state_dict(self, device=None) -> dict:
        return dict(kind="flowmatch_euler.v1", steps=self.steps, shift=self.shift, mu=self.mu,
                    train_steps=self.train_steps, sigmas=self.custom_sigmas, step_index=self.step_index)

    @classmethod
    def from_state_dict(cls, sd: dict, device=None) -> "FlowMatchEulerScheduler":
        if sd.get("kind") != "flowmatch_euler.v1":
            raise ValueError("not a flow-matching Euler scheduler state")
        s = cls(sd["steps"], sd["shift"], sd["mu"], sd["train_steps"], sd.get("sigmas"))
        s.step_index = int(sd["step_index"])
        return s
