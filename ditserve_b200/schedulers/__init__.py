"""Serialisable diffusion solvers.

* ``UniPCFlowScheduler`` — UniPC multistep (Zhao et al., "UniPC: A Unified
  Predictor-Corrector Framework for Fast Sampling of Diffusion Models", 2023)
  in data-prediction form with the B(h) = expm1(h) ("bh2") variant, driven by
  a flow-matching velocity model.  This is the solver recipe the reference
  pins for Wan (workers/ditserve/models/wan/runtime.py:301-304).
* ``DPMSolverFlowScheduler`` — DPM-Solver++ multistep (orders 1-3, midpoint or
  Heun second-order form) over the same flow parameterisation; the alternative
  solver of the Wan family.
* ``FlowMatchEulerScheduler`` — first-order Euler on the flow ODE with the
  static or resolution-dependent ("mu") sigma shift used for SD3.5
  (workers/ditserve/models/sd35.py:841-860).

All produce, per step, the linear coefficients applied by the fused
``ops.sched_step`` kernel (CFG combine + update in one pass), and all can be
captured with ``state_dict()`` and restored bit-exactly with
``load_state_dict()`` (history buffers included).  ``make_scheduler`` builds one
by solver name over a given sigma grid and ``scheduler_from_state`` restores
any of them from its state dict.
"""
from .dpmpp import DPMSolverFlowScheduler
from .flowmatch import FlowMatchEulerScheduler, flow_shift_sigmas, mu_for_seq_len
from .unipc import UniPCFlowScheduler, unipc_flow_sigmas

SOLVERS = ("unipc", "dpm++", "euler")

_KINDS = {"unipc_flow.v1": UniPCFlowScheduler, DPMSolverFlowScheduler.KIND: DPMSolverFlowScheduler,
          "flowmatch_euler.v1": FlowMatchEulerScheduler}


def make_scheduler(solver: str, steps: int, *, sigmas: list[float] | None = None, flow_shift: float = 3.0):
    """A solver by name.  ``sigmas`` (``steps + 1`` values, terminal sigma last) replaces the
    solver's default grid; without it UniPC and DPM-Solver++ walk the flow-shift grid of
    ``unipc_flow_sigmas`` and Euler the shifted linspace of ``flow_shift_sigmas``."""
    if solver == "unipc":
        return UniPCFlowScheduler(steps, flow_shift, sigmas=sigmas)
    if solver == "dpm++":
        return DPMSolverFlowScheduler(steps, flow_shift, sigmas=sigmas)
    if solver == "euler":
        return FlowMatchEulerScheduler(steps, shift=flow_shift, sigmas=sigmas)
    raise ValueError(f"unknown solver {solver!r}; expected one of {SOLVERS}")


def scheduler_from_state(sd: dict, device=None):
    cls = _KINDS.get(sd.get("kind"))
    if cls is None:
        raise ValueError(f"unknown scheduler state kind {sd.get('kind')!r}")
    return cls.from_state_dict(sd, device)


__all__ = ["DPMSolverFlowScheduler", "FlowMatchEulerScheduler", "SOLVERS", "UniPCFlowScheduler",
           "flow_shift_sigmas", "make_scheduler", "mu_for_seq_len", "scheduler_from_state", "unipc_flow_sigmas"]
