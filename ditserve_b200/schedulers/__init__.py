"""Serialisable diffusion solvers.

* ``UniPCFlowScheduler`` — UniPC multistep (Zhao et al., "UniPC: A Unified
  Predictor-Corrector Framework for Fast Sampling of Diffusion Models", 2023)
  in data-prediction form with the B(h) = expm1(h) ("bh2") variant, driven by
  a flow-matching velocity model.  This is the solver recipe the reference
  pins for Wan (workers/ditserve/models/wan/runtime.py:301-304).
* ``FlowMatchEulerScheduler`` — first-order Euler on the flow ODE with the
  static or resolution-dependent ("mu") sigma shift used for SD3.5
  (workers/ditserve/models/sd35.py:841-860).

Both produce, per step, the linear coefficients applied by the fused
``ops.sched_step`` kernel (CFG combine + update in one pass), and both can be
captured with ``state_dict()`` and restored bit-exactly with
``load_state_dict()`` (history buffers included).
"""
from .flowmatch import FlowMatchEulerScheduler, flow_shift_sigmas, mu_for_seq_len
from .unipc import UniPCFlowScheduler, unipc_flow_sigmas

__all__ = ["FlowMatchEulerScheduler", "UniPCFlowScheduler", "flow_shift_sigmas", "mu_for_seq_len",
           "unipc_flow_sigmas"]
