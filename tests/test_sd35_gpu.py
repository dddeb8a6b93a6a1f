"""SD3.5 MMDiT on the sm_100a kernels: packed heterogeneous batch vs individual forwards,
and the GPU result against the fp32 CPU statement of the same (tiny) model."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from ditserve_b200 import ops
from ditserve_b200.models.sd35.model import SD35Config, SD35Transformer

CFG = SD35Config(name="sd3.5-gpu-test", layers=3, heads=24, head_dim=64, joint_dim=512, pooled_dim=256, pos_max=128,
                 dual_layers=(0,))


def _inputs(cfg, dev, dtype):
    g = torch.Generator().manual_seed(0)
    lat = [torch.randn(16, 128, 128, generator=g), torch.randn(16, 64, 64, generator=g)]
    ctx = [torch.randn(333, cfg.joint_dim, generator=g), torch.randn(333, cfg.joint_dim, generator=g)]
    pool = [torch.randn(cfg.pooled_dim, generator=g) for _ in range(2)]
    return ([l.to(dev, dtype) for l in lat], [900.0, 300.0], [c.to(dev, dtype) for c in ctx],
            [p.to(dev, dtype) for p in pool])


def test_sd35_packed_matches_individual_and_cpu_reference():
    dev = torch.device("cuda", 0)
    m = SD35Transformer.random_init(CFG, device=dev, dtype=torch.bfloat16, seed=4)
    lat, t, ctx, pool = _inputs(CFG, dev, torch.bfloat16)
    packed = m.forward_packed(lat, t, ctx, pool)
    ops.check_status(dev)
    for i in range(2):
        solo = m.forward_packed([lat[i]], [t[i]], [ctx[i]], [pool[i]])[0]
        assert torch.equal(packed[i], solo), "packing changed the numerics"
    # fp32 CPU statement of the same weights
    mc = SD35Transformer(CFG)
    mc.load_state_dict({k: v.float().cpu() for k, v in m.state_dict().items()})
    mc.prepare()
    ref = mc.forward_packed([l.float().cpu() for l in lat], t, [c.float().cpu() for c in ctx],
                            [p.float().cpu() for p in pool])
    for a, b in zip(packed, ref):
        a = a.float().cpu()
        rel = ((a - b).norm() / b.norm()).item()
        assert rel < 5e-2, rel
