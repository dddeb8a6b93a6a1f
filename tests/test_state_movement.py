"""Tiered state, two-phase migration with host-side failure injection, inventory/certificates."""
import pytest
import torch

from ditserve_b200.models.migration import (MigrationEndpoint, MigrationError, check_certificate, inventory,
                                            local_roundtrip, migrate, refresh_certificate)
from ditserve_b200.models.tiered import PinnedSlabPool, TieredStore
from ditserve_b200.models.wan.runtime import WanEngine

SPEC = dict(model="wan-tiny", height=64, width=64, frames=13, steps=3, guidance=5.0, seed=4)


def _engine():
    return WanEngine("wan-tiny", device="cpu", dtype=torch.float32, seed=1)


def test_slab_pool_reuses_and_respects_budget():
    pool = PinnedSlabPool(1 << 16, pin=False)
    a = pool.acquire(5000)
    pool.release(a)
    b = pool.acquire(6000)
    assert b is a and pool.stats()["reuses"] == 1
    with pytest.raises(MemoryError):
        pool.acquire(1 << 17)


def test_tiered_offload_prefetch_is_exact():
    e = _engine()
    st = e.prepare(SPEC)
    e.step(st)
    snap = e.snapshot(st, device="cpu")
    store = TieredStore(PinnedSlabPool(64 << 20, pin=False))
    store.offload("r", snap)
    back = store.prefetch("r", device="cpu")
    full = e.run(e.prepare(SPEC))
    resumed = e.restore(back)
    e.run(resumed)
    assert torch.equal(resumed.latents, full.latents)


@pytest.mark.parametrize("fail_after", ["pause", "prepare", "ack"])
def test_migration_aborts_cleanly(fail_after):
    e = _engine()
    st = e.prepare(SPEC)
    e.step(st)
    src, dst = MigrationEndpoint(e, {"r": st}), MigrationEndpoint(e, {})
    with pytest.raises(MigrationError):
        migrate(src, dst, "r", epoch=7, fail_after=fail_after)
    assert "r" in src.states and not src.paused and not dst.pending and "r" not in dst.states
    migrate(src, dst, "r", epoch=8)  # a retry with a new epoch succeeds
    assert "r" not in src.states and "r" in dst.states


def test_migration_mid_step_is_bitwise_and_stale_epochs_are_rejected():
    e = _engine()
    full = e.run(e.prepare(SPEC))
    st = e.prepare(SPEC)
    e.advance(st, blocks=1)  # mid-step continuation packet
    src, dst = MigrationEndpoint(e, {"r": st}), MigrationEndpoint(e, {})
    pkt = src.pause("r", 3)
    dst.prepare("r", 3, pkt["digest"], pkt["packet"])
    with pytest.raises(MigrationError):
        dst.commit("r", 2, pkt["digest"])
    src.release("r", 3, pkt["digest"])
    dst.commit("r", 3, pkt["digest"])
    moved = dst.states["r"]
    while not moved.done:
        e.advance(moved)
    assert torch.equal(moved.latents, full.latents)
    rt = local_roundtrip(e, e.prepare(SPEC))
    assert rt.step == 0


def test_inventory_and_certificates():
    e = _engine()
    st = e.prepare(SPEC)
    e.step(st)
    inv = inventory(st)
    assert inv["tensors"]["latents"]["shape"] == [1, 16, 4, 8, 8] and inv["bytes"] > 0
    cert = refresh_certificate(st, "wan-tiny@1")
    assert check_certificate(st, "wan-tiny@1", cert)
    assert not check_certificate(st, "wan-tiny@2", cert)
    e.step(st)
    assert not check_certificate(st, "wan-tiny@1", cert)
