"""Encoder pool, negative-prompt cache, async/chunked decode through the Wan backend, profiling."""
import torch

from ditserve_b200.models.encoder_pool import EncoderPool, NegativePromptCache, SyntheticEncoder, trim_and_pad


def test_encoder_pool_and_cache(tmp_path):
    pool = EncoderPool(SyntheticEncoder(64), max_len=16, slab_dir=str(tmp_path))
    try:
        t1 = pool.submit("a red kettle on a table", negative="blurry")
        t2 = pool.submit("a red kettle on a table", negative="blurry")
        a, b = pool.fetch(t1, dtype=torch.float32), pool.fetch(t2, dtype=torch.float32)
        assert torch.equal(a["prompt"], b["prompt"]) and a["prompt"].shape == (16, 64)
        assert torch.count_nonzero(a["prompt"][6:]) == 0  # valid tokens kept, padding zero
        assert pool.neg.hits >= 1
    finally:
        pool.close()
    c = NegativePromptCache(max_entries=2, max_bytes=1 << 20)
    for k in "abc":
        c.put(k, torch.zeros(10))
    assert c.get("a") is None and c.get("c") is not None
    x = torch.ones(5, 3)
    assert trim_and_pad(x, 2, 4).sum() == 6


def test_wan_backend_decode_ops(tmp_path):
    from ditserve_b200.models.wan.backend import WanBackend
    w = WanBackend({"model": "wan-tiny", "device": "cpu", "transfer_dir": str(tmp_path)})
    w.prepare(dict(id=1, spec=dict(request_id="v", height=64, width=64, frames=9, steps=1, seed=1)))
    w.advance(dict(id=2, state_id="v", steps=1))
    t = w.decode_start(dict(id=3, state_id="v"))["ticket"]
    out = w.decode_poll(dict(id=4, ticket=t, wait=True, output_mode="digest"))
    assert out["ready"] and out["shape"] == [1, 3, 9, 64, 64]
    t2 = w.decode_start(dict(id=5, state_id="v", chunked=True))["ticket"]
    r = w.decode_poll(dict(id=6, ticket=t2, frames=1, output_mode="digest"))
    while not r["ready"]:
        r = w.decode_poll(dict(id=7, ticket=t2, frames=1, output_mode="digest"))
    assert r["artifact"]["array_sha256"] == out["artifact"]["array_sha256"]


def test_module_timer_and_trace(tmp_path):
    from ditserve_b200.models.wan.runtime import WanEngine
    from ditserve_b200.utils.profiling import ModuleTimer, kineto_trace
    e = WanEngine("wan-tiny", device="cpu", dtype=torch.float32)
    st = e.prepare(dict(model="wan-tiny", height=64, width=64, frames=5, steps=2, seed=1))
    timer = ModuleTimer(e.model)
    e.step(st)
    rep = timer.report()
    timer.close()
    assert set(rep) == {"blocks.0", "blocks.1"}
    rows = kineto_trace(lambda: e.step(st), str(tmp_path / "trace.json"))
    assert isinstance(rows, list)
