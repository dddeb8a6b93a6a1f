"""DPM-Solver++ flow solver: the fused-step coefficients against a textbook float64
restatement, convergence order on an analytic flow, bit-exact resume, and the solver
choice through the Wan and SD3.5 engines (CPU reference path)."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from ditserve_b200.schedulers import (DPMSolverFlowScheduler, FlowMatchEulerScheduler, UniPCFlowScheduler,
                                      make_scheduler, scheduler_from_state, unipc_flow_sigmas)


def lam(s):
    return math.inf if s <= 0 else math.log(1 - s) - math.log(s)


def textbook(sigmas, x, velocity, order, solver_type="midpoint", lower_order_final=True):
    """DPM-Solver++ multistep written in its D0/D1/D2 form, float64 numpy."""
    steps = len(sigmas) - 1
    ms, ss = [], []
    for k in range(steps):
        s0, t = sigmas[k], sigmas[k + 1]
        m0 = x - s0 * velocity(x, s0)
        o = min(order, len(ms) + 1)
        if lower_order_final and steps < 15:
            o = min(o, steps - k)
        if t == 0:
            o = 1
        h = lam(t) - lam(s0)
        a_t = 1 - t
        phi = math.expm1(-h)
        xt = (t / s0) * x - a_t * phi * m0
        if o >= 2:
            r0 = (lam(s0) - lam(ss[-1])) / h
            D1_0 = (m0 - ms[-1]) / r0
            if o == 2:
                xt = xt - 0.5 * a_t * phi * D1_0 if solver_type == "midpoint" else xt + a_t * (phi / h + 1) * D1_0
            else:
                r1 = (lam(ss[-1]) - lam(ss[-2])) / h
                D1_1 = (ms[-1] - ms[-2]) / r1
                D1 = D1_0 + r0 / (r0 + r1) * (D1_0 - D1_1)
                D2 = (D1_0 - D1_1) / (r0 + r1)
                xt = xt + a_t * (phi / h + 1) * D1 - a_t * ((phi + h) / h ** 2 - 0.5) * D2
        ms.append(m0)
        ss.append(s0)
        x = xt
    return x


# Gaussian data x0 ~ N(mu, c^2): the flow marginal at s is N((1-s) mu, (1-s)^2 c^2 + s^2), the
# ideal velocity is (x - E[x0 | x]) / s and the ODE keeps the standardised coordinate fixed.
MU, C = 0.7, 0.5


def ideal_velocity(x, s):
    var = (1 - s) ** 2 * C ** 2 + s ** 2
    x0 = MU + (1 - s) * C ** 2 / var * (x - (1 - s) * MU)
    return (x - x0) / s


def start_and_exact(s0, z):
    return (1 - s0) * MU + math.sqrt((1 - s0) ** 2 * C ** 2 + s0 ** 2) * z, MU + C * z


def run(sched, x):
    xt = torch.tensor(x, dtype=torch.float32)
    while not sched.done:
        s = sched.sigmas[sched.step_index]
        v = torch.tensor(ideal_velocity(xt.double().numpy(), s), dtype=torch.float32)
        sched.step(xt, v)
    return xt.double().numpy()


@pytest.mark.parametrize("order,solver_type", [(1, "midpoint"), (2, "midpoint"), (2, "heun"), (3, "midpoint")])
def test_coefficients_match_textbook(order, solver_type):
    z = np.random.default_rng(0).standard_normal(64)
    for steps in (6, 20):
        sigmas = unipc_flow_sigmas(steps, 3.0)
        x_start, _ = start_and_exact(sigmas[0], z)
        want = textbook(sigmas, x_start, ideal_velocity, order, solver_type)
        got = run(DPMSolverFlowScheduler(steps, 3.0, order=order, solver_type=solver_type), x_start)
        np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-5)


def lambda_grid(steps, s_hi=0.95, s_lo=0.05):
    lams = np.linspace(lam(s_hi), lam(s_lo), steps + 1)
    return [float(1.0 / (1.0 + math.exp(v))) for v in lams]   # s = sigmoid(-lambda)


def marginal(s, z):
    return (1 - s) * MU + math.sqrt((1 - s) ** 2 * C ** 2 + s ** 2) * z


def test_convergence_order():
    # a grid uniform in lambda that stops short of sigma 0, so every step has the full order
    z = np.random.default_rng(1).standard_normal(256)
    errs = {}
    for order in (1, 2, 3):
        for steps in (8, 16, 32):
            grid = lambda_grid(steps)
            sched = DPMSolverFlowScheduler(steps, order=order, lower_order_final=False, sigmas=grid)
            got = run(sched, marginal(grid[0], z))
            errs[(order, steps)] = float(np.abs(got - marginal(grid[-1], z)).max())
    rate = {o: math.log2(errs[(o, 16)] / errs[(o, 32)]) for o in (1, 2, 3)}
    assert 0.8 < rate[1] < 1.3, (rate, errs)
    assert rate[2] > 1.7, (rate, errs)
    assert rate[3] > 2.4 or errs[(3, 32)] < 1e-5, (rate, errs)
    assert errs[(2, 32)] < errs[(1, 32)] / 4


def test_dpmpp_first_order_is_euler_in_data_space_at_final_sigma():
    # a step that lands on sigma 0 returns the data estimate itself
    s = DPMSolverFlowScheduler(1, 3.0)
    x = torch.randn(32)
    v = torch.randn(32)
    want = x - s.sigmas[0] * v
    s.step(x, v)
    torch.testing.assert_close(x, want)


def test_resume_bit_exact_and_registry():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(512, generator=g)
    vs = [torch.randn(512, generator=g) for _ in range(10)]
    for solver in ("unipc", "dpm++", "euler"):
        a = make_scheduler(solver, 10, flow_shift=5.0)
        xa = x.clone()
        for i in range(4):
            a.step(xa, vs[i])
        sd = a.state_dict()
        b = scheduler_from_state(sd)
        assert type(b) is type(a)
        xb = xa.clone()
        for i in range(4, 10):
            a.step(xa, vs[i])
            b.step(xb, vs[i])
        assert torch.equal(xa, xb), solver
    with pytest.raises(ValueError):
        make_scheduler("ddim", 10)
    with pytest.raises(ValueError):
        scheduler_from_state({"kind": "nope"})


def test_custom_grid_is_kept_in_state():
    grid = unipc_flow_sigmas(12, 5.0)
    e = make_scheduler("euler", 12, sigmas=grid)
    assert e.sigmas == grid and isinstance(e, FlowMatchEulerScheduler)
    assert scheduler_from_state(e.state_dict()).sigmas == grid
    u = make_scheduler("unipc", 12, sigmas=[0.9, 0.8, 0.7, 0.6, 0.5, 0.4, 0.3, 0.25, 0.2, 0.1, 0.05, 0.02, 0.0])
    assert isinstance(u, UniPCFlowScheduler) and scheduler_from_state(u.state_dict()).sigmas[0] == 0.9
    with pytest.raises(ValueError):
        make_scheduler("dpm++", 12, sigmas=[0.5, 0.0])


def test_wan_engine_solver_choice_and_restore():
    from ditserve_b200.models.wan.runtime import WanEngine, WanSpec
    eng = WanEngine("wan-tiny", device="cpu", dtype=torch.float32, seed=1)
    base = dict(model="wan-tiny", height=32, width=32, frames=5, steps=4, guidance=3.0, seed=2)
    outs = {}
    for solver in ("unipc", "dpm++", "euler"):
        st = eng.prepare(dict(base, solver=solver))
        eng.step(st)
        eng.step(st)
        st2 = eng.restore(eng.snapshot(st))
        while not st.done:
            eng.step(st)
            eng.step(st2)
        assert st2.done and torch.equal(st.latents, st2.latents), solver
        outs[solver] = st.latents.clone()
    assert not torch.equal(outs["unipc"], outs["dpm++"])
    with pytest.raises(ValueError):
        WanSpec.normalize(dict(base, solver="ddpm"))


def test_sd35_engine_solver_choice():
    from ditserve_b200.models.sd35.model import SD35_TINY
    from ditserve_b200.models.sd35.runtime import SD35Engine
    eng = SD35Engine(SD35_TINY, device="cpu", dtype=torch.float32, seed=2)
    states = [eng.prepare(dict(height=64, width=64, steps=3, guidance=2.0, seed=1, text_len=8, solver=s))
              for s in ("euler", "dpm++")]
    while not all(s.done for s in states):
        eng.advance_batch([s for s in states if not s.done])
    st = eng.prepare(dict(height=64, width=64, steps=4, seed=1, text_len=8, solver="dpm++"))
    eng.advance_batch([st])
    eng.advance_batch([st])
    st2 = eng.restore(eng.snapshot(st))
    while not st.done:
        eng.advance_batch([st, st2])
    torch.testing.assert_close(st.latents, st2.latents, rtol=0, atol=0)
    assert all(torch.isfinite(s.latents).all() for s in states)
    assert not torch.equal(states[0].latents, states[1].latents)
