"""Host-side wiring of the fused peer-memory plans, checked on CPU with the launches faked."""
import pytest
import torch


@pytest.mark.parametrize("steps_done", [0, 2])
def test_fused_cfg_step_reaches_the_cfg_kernel_on_cpu(monkeypatch, steps_done):
    """Host wiring of FusedCFG.fused_step (no GPU): the solver's kernel hook must end in one
    cfg_step_peer launch with this rank's slot, role and solver coefficients."""
    from ditserve_b200.parallel import fused
    from ditserve_b200.schedulers.unipc import UniPCFlowScheduler
    calls = []

    def fake_kernel(name):
        def launch(*args):
            calls.append((name, args))
        return launch
    monkeypatch.setattr(fused, "kernel", fake_kernel)
    monkeypatch.setattr(fused, "status_word", lambda dev: None)

    class FakeGroup:
        channel = 3

        def args(self):
            return 0, [0, 0], 1000

    class FakeHeap:
        def next_epoch(self, ch):
            return 7
    cfgp = object.__new__(fused.FusedCFG)
    n = 64
    cfgp.group, cfgp.heap, cfgp.cfg_size, cfgp.cfg_rank, cfgp.numel = FakeGroup(), FakeHeap(), 2, 1, n
    cfgp.slots = [(0, torch.zeros(n)), (4096, torch.zeros(n))]
    cfgp.calls = 0
    sch = UniPCFlowScheduler(4)
    x = torch.randn(n)
    for _ in range(steps_done):
        sch.step(x, torch.randn(n), None, 1.0)
    mine = torch.randn(n)
    cfgp.fused_step(sch, x, mine, 5.0)
    assert [c[0] for c in calls] == ["cfg_step_peer"]
    args = calls[0][1]
    assert torch.equal(args[0], mine) and args[1] == 0 and args[2] == 1 and args[3] == 5.0
