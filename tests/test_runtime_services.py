"""Host services of the worker runtime (CPU): SM partition math, MPS control gating,
remote bridge over localhost TCP with doorbell mirroring, model integrity, client."""
import json
import os
import stat
import subprocess
import sys
import threading

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_partition_sms():
    from ditserve_b200.runtime.green_context import partition_sms
    assert partition_sms(148, [3, 1]) == [112, 32] or sum(partition_sms(148, [3, 1])) == 144
    s = partition_sms(148, [2, 1, 1])
    assert sum(s) <= 148 and all(x % 8 == 0 and x >= 8 for x in s)
    assert partition_sms(108, [72, 36]) == [72, 32] or sum(partition_sms(108, [72, 36])) <= 108
    with pytest.raises(ValueError):
        partition_sms(16, [1, 1, 1])


def test_mps_control_is_refused_by_default(tmp_path):
    from ditserve_b200.runtime.green_context import mps_control
    fake = tmp_path / "fake-mps"
    log = tmp_path / "calls"
    fake.write_text(f"#!/bin/sh\ncat >> {log}\nexit 0\n")
    fake.chmod(fake.stat().st_mode | stat.S_IEXEC)
    with pytest.raises(PermissionError):
        mps_control({"action": "quit"}, binary=str(fake))
    out = mps_control({"action": "quit"}, binary=str(fake), allowed=True)
    assert out["quit"] and "quit" in log.read_text()


def test_remote_bridge_relays_ops_and_mirrors_doorbells(tmp_path):
    from ditserve_b200.runtime.doorbell import Doorbell
    from ditserve_b200.runtime.remote_bridge import BridgeDaemon
    daemon = BridgeDaemon("127.0.0.1", 0)
    t = threading.Thread(target=daemon.serve_forever, daemon=True)
    t.start()
    cfg = {"options": {"costs": {"step_ms": 400}}}
    proxy = subprocess.Popen([sys.executable, "-m", "ditserve_b200.runtime.remote_bridge", "proxy", "--connect",
                              f"127.0.0.1:{daemon.port}", "--backend", "mock", "--config", json.dumps(cfg)],
                             cwd=ROOT, stdin=subprocess.PIPE, stdout=subprocess.PIPE, text=True)

    def call(i, op, **kw):
        proxy.stdin.write(json.dumps(dict(version=1, id=i, op=op, **kw)) + "\n")
        proxy.stdin.flush()
        return json.loads(proxy.stdout.readline())

    try:
        assert call(1, "hello")["ok"]
        assert call(2, "prepare", spec=dict(request_id="r", steps=1, blocks_per_step=8, seed=0))["ok"]
        bell = Doorbell(str(tmp_path / "bell0"), create=True)
        timer = threading.Timer(0.25, lambda: bell.ring(1))
        timer.start()
        r = call(3, "advance", state_id="r", quantum="step", check_blocks=1, doorbell=dict(path=bell.path, epoch=0))
        assert r["ok"] and r["result"]["doorbell_stop"], r
        assert r["result"]["executed"] < 8
    finally:
        proxy.stdin.close()
        proxy.wait(timeout=10)
        daemon.stop()


def test_remote_bridge_moves_packets_between_nodes(tmp_path):
    """A continuation packet crosses the bridge both ways: a remote export lands in the
    proxy's staging directory, a local packet is pushed into the remote session for import,
    and the run ends bit-identical to an unmoved one.  File staging stays inside the session."""
    from ditserve_b200.models.wan.backend import WanBackend
    from ditserve_b200.runtime.remote_bridge import BridgeDaemon, BridgeProxy
    daemon = BridgeDaemon("127.0.0.1", 0, workdir=str(tmp_path / "node1"))
    threading.Thread(target=daemon.serve_forever, daemon=True).start()
    stage = tmp_path / "stage"
    stage.mkdir()
    proxy = BridgeProxy(f"127.0.0.1:{daemon.port}", "wan", {"model": "wan-tiny", "device": "cpu"},
                        env={"CUDA_VISIBLE_DEVICES": "", "PATH_NOT_PASSED": "x"}, stage_dir=str(stage))
    ids = iter(range(1, 1000))

    def call(op, **kw):
        rep = json.loads(proxy.relay(json.dumps(dict(version=1, id=next(ids), op=op, **kw)) + "\n"))
        assert rep["ok"], rep
        return rep["result"]

    spec = dict(request_id="v", height=64, width=64, frames=5, steps=3, seed=5)
    try:
        call("hello")
        call("prepare", spec=spec)
        call("advance", state_id="v", quantum="step")
        pk = call("block_export", state_id="v")
        assert pk["path"].startswith(str(stage)) and os.path.getsize(pk["path"]) == pk["bytes"]
        call("release", state_id="v")
        local = WanBackend({"model": "wan-tiny", "device": "cpu", "transfer_dir": str(tmp_path)})
        local.block_import(dict(id=1, state_id="v", path=pk["path"], manifest=pk["manifest"]))
        assert not os.path.exists(pk["path"])               # single-use packet consumed
        local.advance(dict(id=2, state_id="v", quantum="step"))
        back = local.block_export(dict(id=3, state_id="v"))
        r = call("block_import", state_id="v", path=back["path"], manifest=back["manifest"])
        assert r["progress"]["step"] == 2 and not os.path.exists(back["path"])
        call("advance", state_id="v", quantum="step")
        moved = call("finish", state_id="v", output_mode="digest")["value"]
        # the file frames cannot reach outside the session directory
        with pytest.raises(OSError):
            proxy.pull_file(str(tmp_path / "stage" / "nothing"))
        with pytest.raises(OSError):
            proxy._call({"bridge": "put_file", "name": "../escape", "data_b64": ""}, "put_file")
    finally:
        proxy.close()
        daemon.stop()
    ref = WanBackend({"model": "wan-tiny", "device": "cpu", "transfer_dir": str(tmp_path)})
    ref.prepare(dict(id=1, spec=spec))
    ref.advance(dict(id=2, state_id="v", steps=3))
    assert ref.finish(dict(id=3, state_id="v", output_mode="digest"))["value"] == moved


def test_snapshot_integrity(tmp_path):
    from ditserve_b200.runtime.model_integrity import IntegrityError, build_manifest, verify_snapshot
    (tmp_path / "transformer").mkdir()
    (tmp_path / "transformer" / "a.bin").write_bytes(b"abc")
    (tmp_path / "model_index.json").write_text("{}")
    man = build_manifest(tmp_path)
    assert verify_snapshot(tmp_path, man)["verified"]
    (tmp_path / "transformer" / "a.bin").write_bytes(b"abd")
    with pytest.raises(IntegrityError):
        verify_snapshot(tmp_path, man)


def test_diffusers_layout_round_trip(tmp_path):
    import torch
    from safetensors.torch import save_file
    from ditserve_b200.models.wan.config import WAN_TINY
    from ditserve_b200.models.wan.model import WanTransformer
    from ditserve_b200.runtime.model_integrity import load_diffusers_transformer
    a = WanTransformer.random_init(WAN_TINY, dtype=torch.float32, seed=1)
    (tmp_path / "transformer").mkdir()
    save_file({k: v.contiguous() for k, v in a.state_dict().items()},
              str(tmp_path / "transformer" / "diffusion_pytorch_model.safetensors"))
    b = WanTransformer.random_init(WAN_TINY, dtype=torch.float32, seed=2)
    info = load_diffusers_transformer(b, tmp_path)
    assert info["tensors"] == len(a.state_dict())
    for k, v in a.state_dict().items():
        assert torch.equal(v, b.state_dict()[k])


def test_remote_bridge_refuses_a_wrong_token(tmp_path):
    from ditserve_b200.runtime.remote_bridge import BridgeDaemon, BridgeProxy
    daemon = BridgeDaemon("127.0.0.1", 0, workdir=str(tmp_path), token="s3cret")
    threading.Thread(target=daemon.serve_forever, daemon=True).start()
    try:
        bad = BridgeProxy(f"127.0.0.1:{daemon.port}", "mock", {}, token="wrong", stage_dir=str(tmp_path))
        with pytest.raises((ConnectionError, OSError)):
            bad.relay(json.dumps(dict(version=1, id=1, op="hello")) + "\n")
        bad.close()
        good = BridgeProxy(f"127.0.0.1:{daemon.port}", "mock", {}, token="s3cret", stage_dir=str(tmp_path))
        assert json.loads(good.relay(json.dumps(dict(version=1, id=1, op="hello")) + "\n"))["ok"]
        good.close()
    finally:
        daemon.stop()


def test_remote_bridge_refuses_public_listen_without_token(monkeypatch):
    """Off the loopback interface the daemon would start workers for anyone: no token, no daemon."""
    from ditserve_b200.runtime.remote_bridge import BridgeDaemon, _is_loopback
    monkeypatch.delenv("DITSERVE_BRIDGE_TOKEN", raising=False)
    assert _is_loopback("127.0.0.1") and _is_loopback("localhost")
    assert not _is_loopback("0.0.0.0")
    with pytest.raises(ValueError, match="without a token"):
        BridgeDaemon("0.0.0.0", 0)
    d = BridgeDaemon("0.0.0.0", 0, token="s3cret")  # with a shared secret it may listen anywhere
    d.stop()


def test_remote_bridge_file_frames_stay_in_the_session(tmp_path):
    """A client that names its own transfer_dir still cannot read or delete files outside the
    session directory: the worker's transfer_dir is replaced and get_file is confined."""
    from ditserve_b200.runtime.remote_bridge import BridgeDaemon, BridgeProxy
    outside = tmp_path / "outside"
    outside.mkdir()
    secret = outside / "keep.txt"
    secret.write_text("not yours")
    daemon = BridgeDaemon("127.0.0.1", 0, workdir=str(tmp_path / "node1"))
    threading.Thread(target=daemon.serve_forever, daemon=True).start()
    try:
        proxy = BridgeProxy(f"127.0.0.1:{daemon.port}", "mock", {"transfer_dir": str(outside)},
                            stage_dir=str(tmp_path))
        assert json.loads(proxy.relay(json.dumps(dict(version=1, id=1, op="hello")) + "\n"))["ok"]
        with pytest.raises(OSError):
            proxy.pull_file(str(secret), unlink=True)
        assert secret.read_text() == "not yours"
        proxy.close()
    finally:
        daemon.stop()
