"""Worker protocol v1 and the mock backend (CPU, real subprocess framing)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def spawn(backend="mock", config=None):
    return subprocess.Popen([sys.executable, "-m", "ditserve_b200.runtime.worker", "--backend", backend,
                             "--config", json.dumps(config or {})], cwd=ROOT, stdin=subprocess.PIPE,
                            stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)


def call(p, rid, op, **kw):
    p.stdin.write(json.dumps(dict(version=1, id=rid, op=op, **kw)) + "\n")
    p.stdin.flush()
    return json.loads(p.stdout.readline())


def test_envelope_and_strictness():
    p = spawn(config={"options": {"print": "stdout pollution"}})
    try:
        r = call(p, 1, "hello")
        assert r["ok"] and r["result"]["backend"] == "mock" and r["id"] == 1
        p.stdin.write('{"version":1,"id":2,"op":"hello","x":NaN}\n')
        p.stdin.flush()
        bad = json.loads(p.stdout.readline())
        assert bad["ok"] is False and "non-finite" in bad["error"]
        p.stdin.write("not json\n")
        p.stdin.flush()
        assert json.loads(p.stdout.readline())["ok"] is False
        r = call(p, 3, "prepare", spec={"request_id": "a", "steps": 3, "seed": 1})
        assert r["ok"], r  # the injected print went to stderr, framing intact
        r = call(p, 4, "nope")
        assert not r["ok"]
        assert call(p, 5, "shutdown")["ok"]
    finally:
        p.kill()


def test_mock_segmented_equals_uninterrupted():
    from ditserve_b200.models.mock import MockBackend
    b = MockBackend({})
    b.prepare(dict(id=1, spec=dict(request_id="x", steps=4, blocks_per_step=3, seed=5)))
    b.prepare(dict(id=2, spec=dict(request_id="y", steps=4, blocks_per_step=3, seed=5)))
    while b.states["x"]["step"] < 4:
        b.advance(dict(id=3, state_id="x", quantum="step"))
    for n in (1, 2, 1, 1, 3, 2, 2):
        if b.states["y"]["step"] >= 4:
            break
        b.advance(dict(id=4, state_id="y", blocks=n))
    while b.states["y"]["step"] < 4:
        b.advance(dict(id=5, state_id="y", quantum="step"))
    assert b.states["x"]["value"] == b.states["y"]["value"]


def test_mock_export_import_and_tamper():
    from ditserve_b200.models.mock import MockBackend
    a, c = MockBackend({}), MockBackend({})
    a.prepare(dict(id=1, spec=dict(request_id="r", steps=3, blocks_per_step=2, seed=2)))
    a.advance(dict(id=2, state_id="r", blocks=1))
    pk = a.block_export(dict(id=3, state_id="r"))
    with pytest.raises(ValueError, match="manifest"):
        c.block_import(dict(id=4, packet=pk["packet"].replace('"step": 0', '"step": 1'), manifest=pk["manifest"]))
    c.block_import(dict(id=5, packet=pk["packet"], manifest=pk["manifest"]))
    assert c.states["r"]["unit"] == 1


def test_fault_injection_and_doorbell(tmp_path):
    from ditserve_b200.models.mock import MockBackend
    from ditserve_b200.runtime.doorbell import Doorbell
    b = MockBackend({"options": {"fail_ops": ["finish"]}})
    b.prepare(dict(id=1, spec=dict(request_id="r", steps=1, seed=0)))
    b.advance(dict(id=2, state_id="r"))
    with pytest.raises(RuntimeError, match="injected"):
        b.finish(dict(id=3, state_id="r"))
    bell = Doorbell(str(tmp_path / "bell"), create=True)
    b2 = MockBackend({})
    b2.prepare(dict(id=1, spec=dict(request_id="s", steps=2, blocks_per_step=8, seed=0)))
    bell.ring(5)
    r = b2.advance(dict(id=2, state_id="s", quantum="step", check_blocks=2,
                        doorbell=dict(path=bell.path, epoch=4)))
    assert r["doorbell_stop"] and r["executed"] == 2


def test_wan_and_sd35_backends_on_cpu(tmp_path):
    """The model backends speak the same op surface as the mock (tiny models, CPU)."""
    from ditserve_b200.models.sd35.backend import SD35Backend
    from ditserve_b200.models.wan.backend import WanBackend
    w = WanBackend({"model": "wan-tiny", "device": "cpu", "transfer_dir": str(tmp_path)})
    spec = dict(request_id="v", height=64, width=64, frames=13, steps=2, seed=1)
    w.prepare(dict(id=1, spec=spec))
    r = w.advance(dict(id=2, state_id="v", blocks=1))
    assert r["progress"]["block"] == 1
    pk = w.block_export(dict(id=3, state_id="v"))
    w.release(dict(state_id="v"))
    w.block_import(dict(id=4, state_id="v", path=pk["path"], manifest=pk["manifest"]))
    while not w.states["v"].done:
        w.advance(dict(id=5, state_id="v", quantum="step"))
    out = w.finish(dict(id=6, state_id="v", output_mode="digest"))
    w2 = WanBackend({"model": "wan-tiny", "device": "cpu"})
    w2.prepare(dict(id=1, spec=spec))
    w2.advance(dict(id=2, state_id="v", steps=2))
    assert w2.finish(dict(id=3, state_id="v", output_mode="digest"))["value"] == out["value"]
    s = SD35Backend({"model": "sd3.5-tiny", "device": "cpu"})
    for k in ("a", "b"):
        s.prepare(dict(id=1, spec=dict(request_id=k, height=64, width=64, steps=2, seed=3)))
    s.advance_batch(dict(id=2, state_ids=["a", "b"]))
    s.advance_batch(dict(id=3, state_ids=["a", "b"]))
    fa = s.finish(dict(id=4, state_id="a", output_mode="digest"))
    fb = s.finish(dict(id=5, state_id="b", output_mode="digest"))
    assert fa["value"] == fb["value"]  # same seed and spec
