"""ditserve_b200: a Blackwell-native (sm_100a) diffusion-transformer serving framework.

Layers (bottom up):
  ops/          hand-written sm_100a kernels (tcgen05 GEMM + attention, fused norms, solver step)
  parallel/     CFG / Ulysses / ring layouts, symmetric-memory runtime, fused comm kernels
  models/       Wan2.1 / Wan2.2 / SD3.5 DiTs, request state, block executor, backends
  schedulers/   UniPC (flow prediction, bh2) and flow-matching Euler with serialisable state
  runtime/      JSON-lines worker server and its host-side services
The C++ controller (cpp/controller) drives the workers over the JSON-lines protocol.
"""
__version__ = "0.1.0"
