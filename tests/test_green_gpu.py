"""Green Context SM partitions on one GPU: two roles, each with its own stream; work on both
streams completes and matches the same work on the default stream."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_green_pool_two_roles_run_work():
    from ditserve_b200.runtime.green_context import GreenPool
    pool = GreenPool(0, {"video": 112, "image": 36})
    try:
        st = pool.status()
        assert st["sm_counts"]["video"] >= 112 and st["sm_counts"]["image"] >= 8
        assert sum(st["sm_counts"].values()) <= st["total_sms"]
        a = torch.randn(1024, 1024, device="cuda")
        want = a @ a
        outs = {}
        for role in ("video", "image"):
            with torch.cuda.stream(pool.stream(role)):
                outs[role] = a @ a
            pool.stream(role).synchronize()
        for role, o in outs.items():
            assert torch.allclose(o, want, rtol=1e-4, atol=1e-3), role
    finally:
        torch.cuda.synchronize()
        pool.close()
