"""The C++ multi-GPU cluster executor on CPU: mock workers with pairs, continuous image
batches and host-staged regroups; Wan-tiny workers as a gloo world (every member of a
group runs the quantum under its CFG x SP layout, regroups broadcast the state)."""
import json
import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CTL = os.path.join(ROOT, "cpp", "controller")
BUILD = os.path.join(CTL, "build")
BIN = os.path.join(BUILD, "ditserve-b200")


@pytest.fixture(scope="module")
def controller():
    if shutil.which("cmake") is None:
        pytest.skip("cmake unavailable")
    subprocess.run(["cmake", "-S", CTL, "-B", BUILD, "-DCMAKE_BUILD_TYPE=Release"], check=True, capture_output=True)
    subprocess.run(["cmake", "--build", BUILD, "-j", str(os.cpu_count() or 4)], check=True, capture_output=True)
    return BIN


def _run(controller, cfg, tmp_path, allow_gpu=False, timeout=900):
    path = tmp_path / "study.json"
    path.write_text(json.dumps(cfg))
    env = dict(os.environ, DITSERVE_PYTHON=sys.executable, DITSERVE_PACKAGE_ROOT=ROOT)
    cmd = [controller, "--json", "run", "--config", str(path), "--run-id", "c", "--work-dir", str(tmp_path)]
    if allow_gpu:
        cmd.append("--allow-gpu")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=timeout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    rep = json.loads(r.stdout)
    res = json.loads((tmp_path / "c" / "phases" / "cluster" / "result.json").read_text()) \
        if (tmp_path / "c" / "phases" / "cluster" / "result.json").exists() else None
    return rep, res


def _last(rep):
    return rep["phases"]["cluster"]["cells"][-1]["result"]


BUDGET = {"limit_gpu_seconds": 3600, "watchdog_seconds": 900, "repair_reserve_gpu_seconds": 60, "carry": "none"}


def test_mock_cluster_pairs_batches_regroups(controller, tmp_path):
    cfg = {"schema": "ditserve-b200.study.v1", "experiment": "exec-mock",
           "workers": {"vid": {"backend": "mock", "config": {"options": {"costs": {"step_ms": 15},
                                                                          "decode_delay_ms": 20}}},
                       "img": {"backend": "mock", "config": {"options": {"costs": {"step_ms": 5}}}}},
           "budget": BUDGET,
           "phases": [{"id": "cluster", "kind": "cluster", "gpus": 4, "policy": "ditserve", "distributed": True,
                       "workers": {"video": "vid", "image": "img"}, "decode": True,
                       "warmup_forms": "auto", "warmup_image_spec": {"steps": 1},
                       "sp_transport": "export",
                       "options": {"pairing": True, "continuous_batch": 4},
                       "generator": {"count": 12, "seed": 2, "pattern": "poisson", "rate_rps": 40, "classes": [
                           {"weight": 1, "kind": "video", "class": "wan21_480p", "service_ms": 1500,
                            "slo_scale": 4, "spec": {"steps": 4, "blocks_per_step": 3}},
                           {"weight": 2, "kind": "image", "class": "sd35_512", "service_ms": 300, "slo_scale": 4,
                            "spec": {"steps": 3}}]},
                       "gates": [{"pointer": "/last/summary/completed", "op": "==", "value": 12},
                                 {"pointer": "/last/counters/cleanup_verified", "op": "==", "value": True}]}]}
    rep, _ = _run(controller, cfg, tmp_path)
    assert rep["phases"]["cluster"]["gates"]["pass"], rep["phases"]["cluster"]
    last = _last(rep)
    assert last is not None and not last["failures"]
    assert last["counters"]["quanta"] >= 12 and last["trace"]
    assert last["decisions"] and all(len(d["ranking"]) <= 64 for d in last["decisions"])
    assert {"request_id", "laxity_ms", "feasible"} <= set(last["decisions"][0]["ranking"][0])
    # every video's digest equals the 4-step chain of its own seed: copies stayed consistent
    digests = {r["request_id"]: r.get("digest") for r in last["rows"]}
    assert all(digests.values())


def test_wan_tiny_gloo_world_cluster(controller, tmp_path):
    cfg = {"schema": "ditserve-b200.study.v1", "experiment": "exec-wan-gloo",
           "workers": {"wan": {"backend": "wan", "config": {"model": "wan-tiny", "device": "cpu",
                                                            "transfer_dir": str(tmp_path)}}},
           "budget": BUDGET,
           "phases": [{"id": "cluster", "kind": "cluster", "gpus": 2, "policy": "ditserve", "worker": "wan",
                       "distributed": True, "sp_transport": "collective", "collectives": "nccl",
                       "warmup_forms": ["cfg2", "sp2"], "warmup_spec": {"height": 64, "width": 64, "frames": 5},
                       "decode": True,
                       "dist_port": 29000 + os.getpid() % 1000,
                       "generator": {"count": 3, "seed": 4, "pattern": "poisson", "rate_rps": 50, "classes": [
                           {"weight": 1, "kind": "video", "class": "wan21_480p", "service_ms": 20000,
                            "slo_scale": 5, "spec": {"height": 64, "width": 64, "frames": 5, "steps": 3,
                                                     "guidance": 5.0}}]},
                       "gates": [{"pointer": "/last/summary/completed", "op": "==", "value": 3}]}]}
    rep, _ = _run(controller, cfg, tmp_path, allow_gpu=True)
    assert rep["phases"]["cluster"]["gates"]["pass"], rep["phases"]["cluster"]
    last = _last(rep)
    assert not last["failures"], last["failures"]
    assert last["controller_timing"]["warmup_ms"] > 0
    forms = {t["form"] for t in last["trace"]}
    assert forms & {"cfg2", "sp2"}, forms  # at least one quantum ran on both ranks
    assert any(t["quantum"] == "finish" for t in last["trace"])  # VAE decode quanta ran
    assert all(r.get("digest") for r in last["rows"])


def test_cfg_fission_gloo_world(controller, tmp_path):
    """ditserve-approx hands the unconditional rank away while a video's steps run folded."""
    cfg = {"schema": "ditserve-b200.study.v1", "experiment": "exec-fission",
           "workers": {"wan": {"backend": "wan", "config": {"model": "wan-tiny", "device": "cpu",
                                                            "transfer_dir": str(tmp_path)}}},
           "budget": BUDGET,
           "phases": [{"id": "cluster", "kind": "cluster", "gpus": 2, "policy": "ditserve-approx", "worker": "wan",
                       "distributed": True, "sp_transport": "collective", "collectives": "nccl",
                       "dist_port": 28000 + os.getpid() % 1000,
                       "generator": {"count": 1, "seed": 4, "pattern": "offline_all", "classes": [
                           {"weight": 1, "kind": "video", "class": "wan21_480p", "service_ms": 20000,
                            "slo_scale": 5, "spec": {"height": 64, "width": 64, "frames": 5, "steps": 6,
                                                     "guidance": 5.0,
                                                     "cfg_fold": {"warm_frac": 0.0, "threshold": 10.0,
                                                                  "fold_span": 1}}}]},
                       "gates": [{"pointer": "/last/summary/completed", "op": "==", "value": 1}]}]}
    rep, _ = _run(controller, cfg, tmp_path, allow_gpu=True)
    assert rep["phases"]["cluster"]["gates"]["pass"], rep["phases"]["cluster"]
    last = _last(rep)
    assert not last["failures"], last["failures"]
    forms = [t["form"] for t in last["trace"]]
    assert "cfg2" in forms and "sp1" in forms, forms       # full steps on the pair, folded ones alone
    assert last["counters"]["transfers"] >= 1              # the pair regrouped after a folded step


def _guard_cfg(tmp):
    return {"schema": "ditserve-b200.study.v1", "experiment": "exec-guard",
            "workers": {"model": {"backend": "mock", "config": {"options": {"costs": {"step_ms": 40}}}}},
            "budget": BUDGET,
            "phases": [{"id": "cluster", "kind": "cluster", "gpus": 2, "policy": "ditserve",
                        "occupancy_guard": True, "occupancy_interval_ms": 50, "admission_wait_s": 1,
                        "generator": {"count": 3, "seed": 1, "pattern": "offline_all", "classes": [
                            {"kind": "video", "class": "wan21_480p", "service_ms": 5000, "slo_scale": 5,
                             "spec": {"steps": 6, "blocks_per_step": 2}}]}}]}


@pytest.mark.parametrize("table,aborts", [({}, None), ({"1": [{"pid": 999999, "used_mib": "100"}]}, "foreign"),
                                          ("fail", "unknown")])
def test_occupancy_guard(controller, tmp_path, table, aborts):
    path = tmp_path / "occ.json"
    path.write_text(json.dumps(table))
    env = dict(os.environ, DITSERVE_PYTHON=sys.executable, DITSERVE_PACKAGE_ROOT=ROOT,
               DITSERVE_OCCUPANCY_TABLE=str(path))
    cfgp = tmp_path / "study.json"
    cfgp.write_text(json.dumps(_guard_cfg(tmp_path)))
    r = subprocess.run([controller, "--json", "run", "--config", str(cfgp), "--run-id", "g", "--work-dir",
                        str(tmp_path)], capture_output=True, text=True, env=env, timeout=600)
    rep = json.loads(r.stdout)
    last = rep["phases"]["cluster"]["cells"][-1]["result"]
    if aborts is None:
        assert last["occupancy_probes"]
        assert "aborted" not in last and last["summary"]["completed"] == 3
        assert {"prepare", "advance", "finish"} <= {s["stage"] for s in last["spans"]}
    else:
        assert "admission" in last["aborted"] and last["failures"]   # never admitted: GPUs not idle
        assert all(row["status"] in ("done", "failed") for row in last["rows"])


def test_occupancy_guard_aborts_mid_run(controller, tmp_path):
    """A foreign process appearing on one of the phase's GPUs after admission aborts the phase."""
    import time
    path = tmp_path / "occ.json"
    path.write_text("{}")
    cfg = _guard_cfg(tmp_path)
    cfg["phases"][0]["generator"]["count"] = 6
    cfg["phases"][0]["generator"]["classes"][0]["spec"]["steps"] = 40
    cfgp = tmp_path / "study.json"
    cfgp.write_text(json.dumps(cfg))
    env = dict(os.environ, DITSERVE_PYTHON=sys.executable, DITSERVE_PACKAGE_ROOT=ROOT,
               DITSERVE_OCCUPANCY_TABLE=str(path))
    p = subprocess.Popen([controller, "--json", "run", "--config", str(cfgp), "--run-id", "m", "--work-dir",
                          str(tmp_path)], stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, env=env)
    log = tmp_path / "m" / "video0.log"
    deadline = time.time() + 120
    while time.time() < deadline and not (log.exists() and log.stat().st_size >= 0 and (tmp_path / "m").exists()):
        time.sleep(0.1)
    time.sleep(3.0)  # workers up, trace running
    path.write_text(json.dumps({"0": [{"pid": 999999, "used_mib": "10"}]}))
    out, err = p.communicate(timeout=600)
    rep = json.loads(out)
    last = rep["phases"]["cluster"]["cells"][-1]["result"]
    assert "foreign GPU process" in last.get("aborted", ""), (last.get("aborted"), last["summary"])
    assert last["failures"] and any(pr["state"] == "busy" for pr in last["occupancy_probes"])


@pytest.fixture()
def bridge_daemon(tmp_path):
    """A bridge daemon on 127.0.0.1 standing in for a second node."""
    env = dict(os.environ, PYTHONPATH=ROOT)
    p = subprocess.Popen([sys.executable, "-m", "ditserve_b200.runtime.remote_bridge", "daemon", "--listen",
                          "127.0.0.1:0"], stdout=subprocess.PIPE, text=True, env=env, cwd=str(tmp_path))
    try:
        port = json.loads(p.stdout.readline())["listening"]
        yield f"127.0.0.1:{port}"
    finally:
        p.terminate()
        p.wait(timeout=10)


def test_remote_slot_through_bridge(controller, tmp_path, bridge_daemon):
    """Slot 1's workers live on 'another node' behind the bridge; requests placed there run
    there, and continuation packets move between the local and the remote slot."""
    cfg = {"schema": "ditserve-b200.study.v1", "experiment": "exec-remote",
           "workers": {"wan": {"backend": "wan", "config": {"model": "wan-tiny", "device": "cpu",
                                                            "transfer_dir": str(tmp_path)}}},
           "budget": BUDGET,
           "phases": [{"id": "cluster", "kind": "cluster", "gpus": 2, "policy": "ditserve", "worker": "wan",
                       "remote_slots": {"1": {"address": bridge_daemon, "device": "0"}},
                       "options": {"forms": ["sp1"]},
                       "generator": {"count": 8, "seed": 3, "pattern": "poisson", "rate_rps": 20, "classes": [
                           {"weight": 1, "kind": "video", "class": "wan21_480p", "service_ms": 3000,
                            "slo_scale": 3, "spec": {"height": 64, "width": 64, "frames": 5, "steps": 4,
                                                     "guidance": 5.0}},
                           {"weight": 1, "kind": "video", "class": "wan21_480p", "service_ms": 300,
                            "slo_scale": 2, "spec": {"height": 32, "width": 32, "frames": 1, "steps": 2,
                                                     "guidance": 5.0}}]},
                       "gates": [{"pointer": "/last/summary/completed", "op": "==", "value": 8}]}]}
    rep, _ = _run(controller, cfg, tmp_path, allow_gpu=True)
    assert rep["phases"]["cluster"]["gates"]["pass"], rep["phases"]["cluster"]
    last = _last(rep)
    assert not last["failures"], last["failures"]
    groups = [t.get("group") or t.get("gpus") for t in last["trace"]]
    assert any(1 in (g or []) for g in groups), groups
    # every output equals an unmoved local run of its spec, wherever its quanta ran
    from ditserve_b200.models.wan.backend import WanBackend
    ref = WanBackend({"model": "wan-tiny", "device": "cpu", "transfer_dir": str(tmp_path)})
    for i, row in enumerate(last["rows"]):
        spec = dict(row["spec"], request_id=f"ref{i}")
        ref.prepare(dict(id=1, spec=spec))
        ref.advance(dict(id=2, state_id=f"ref{i}", steps=spec["steps"]))
        want = ref.finish(dict(id=3, state_id=f"ref{i}", output_mode="digest"))["value"]
        assert row["digest"] == want, row


@pytest.mark.parametrize("foreign", [True, False])
def test_occupancy_guard_covers_remote_slots(controller, tmp_path, foreign):
    """A foreign process on a remote slot's GPU (reported by that node's daemon) aborts the phase;
    an idle remote node lets it run."""
    table = tmp_path / "occ.json"
    table.write_text(json.dumps({"0": [{"pid": 999999, "used_mib": "100"}]} if foreign else {}))
    env = dict(os.environ, PYTHONPATH=ROOT, DITSERVE_OCCUPANCY_TABLE=str(table))
    d = subprocess.Popen([sys.executable, "-m", "ditserve_b200.runtime.remote_bridge", "daemon", "--listen",
                          "127.0.0.1:0"], stdout=subprocess.PIPE, text=True, env=env, cwd=str(tmp_path))
    try:
        port = json.loads(d.stdout.readline())["listening"]
        cfg = _guard_cfg(tmp_path)
        ph = cfg["phases"][0]
        ph["remote_slots"] = {"1": {"address": f"127.0.0.1:{port}", "device": "0"}}
        ph["admission_wait_s"] = 1
        path = tmp_path / "study.json"
        path.write_text(json.dumps(cfg))
        run_env = dict(os.environ, DITSERVE_PYTHON=sys.executable, DITSERVE_PACKAGE_ROOT=ROOT)
        empty = tmp_path / "local.json"
        empty.write_text("{}")
        run_env["DITSERVE_OCCUPANCY_TABLE"] = str(empty)  # this node: idle
        r = subprocess.run([controller, "--json", "run", "--config", str(path), "--run-id", "g", "--work-dir",
                            str(tmp_path)], capture_output=True, text=True, env=run_env, timeout=600)
        rep = json.loads(r.stdout)
        last = rep["phases"]["cluster"]["cells"][-1]["result"]
        if foreign:
            assert "admission" in last.get("aborted", ""), {k: last.get(k) for k in ("aborted", "occupancy_probes")}
            assert last["failures"]
        else:
            assert "aborted" not in last and last["summary"]["completed"] == 3
    finally:
        d.terminate()
        d.wait(timeout=10)


def test_two_node_worlds_through_the_bridge(controller, tmp_path, bridge_daemon):
    """Slots 0-1 on this node and 2-3 behind a bridge daemon ("another node") each form their own
    Gloo world of Wan-tiny workers; groups never cross nodes (degrees capped at the node size) and
    every request completes."""
    cfg = {"schema": "ditserve-b200.study.v1", "experiment": "exec-two-node",
           "workers": {"wan": {"backend": "wan", "config": {"model": "wan-tiny", "device": "cpu",
                                                            "transfer_dir": str(tmp_path)}}},
           "budget": BUDGET,
           "phases": [{"id": "cluster", "kind": "cluster", "gpus": 4, "policy": "ditserve", "worker": "wan",
                       "distributed": True, "sp_transport": "collective", "collectives": "nccl",
                       "remote_slots": {"2": {"address": bridge_daemon, "device": "0"},
                                        "3": {"address": bridge_daemon, "device": "1"}},
                       "dist_port": 27000 + os.getpid() % 1000,
                       "generator": {"count": 4, "seed": 6, "pattern": "offline_all", "classes": [
                           {"weight": 1, "kind": "video", "class": "wan21_480p", "service_ms": 20000,
                            "slo_scale": 5, "spec": {"height": 64, "width": 64, "frames": 5, "steps": 2,
                                                     "guidance": 5.0}}]},
                       "gates": [{"pointer": "/last/summary/completed", "op": "==", "value": 4}]}]}
    rep, _ = _run(controller, cfg, tmp_path, allow_gpu=True)
    assert rep["phases"]["cluster"]["gates"]["pass"], rep["phases"]["cluster"]
    last = _last(rep)
    assert not last["failures"], last["failures"]
    groups = [tuple(t.get("group") or []) for t in last["trace"]]
    assert all(set(g) <= {0, 1} or set(g) <= {2, 3} for g in groups), groups
    assert any(set(g) == {2, 3} for g in groups), groups       # the remote node ran a 2-rank group
    assert all(r.get("digest") for r in last["rows"])  # CFG2 groups: equal up to the drift gate, not bitwise


def test_patch_parallel_decode_in_a_gloo_world(controller, tmp_path):
    """decode_parallel: a finished video decodes on the group of its last step, every member
    decoding its rows with halo exchange (the row-split decode equals the single-rank one to
    fp32 rounding: tests/test_wan_vae_fast.py), and every member ends with the same video."""
    def study(parallel, port):
        return {"schema": "ditserve-b200.study.v1", "experiment": f"exec-ppdecode-{parallel}",
                "workers": {"wan": {"backend": "wan", "config": {"model": "wan-tiny", "device": "cpu",
                                                                 "transfer_dir": str(tmp_path)}}},
                "budget": BUDGET,
                "phases": [{"id": "cluster", "kind": "cluster", "gpus": 2, "policy": "static-sp2", "worker": "wan",
                            "distributed": True, "sp_transport": "collective", "collectives": "nccl",
                            "decode": True, "decode_parallel": parallel, "dist_port": port,
                            "generator": {"count": 1, "seed": 4, "pattern": "offline_all", "classes": [
                                {"weight": 1, "kind": "video", "class": "wan21_480p", "service_ms": 20000,
                                 "slo_scale": 5, "spec": {"height": 64, "width": 64, "frames": 5, "steps": 2,
                                                          "guidance": 5.0}}]},
                            "gates": [{"pointer": "/last/summary/completed", "op": "==", "value": 1}]}]}
    base = 30000 + os.getpid() % 1000
    for parallel in (False, True):
        sub = tmp_path / ("pp" if parallel else "single")
        sub.mkdir()
        rep, _ = _run(controller, study(parallel, base + (7 if parallel else 0)), sub, allow_gpu=True)
        assert rep["phases"]["cluster"]["gates"]["pass"], rep["phases"]["cluster"]
        last = _last(rep)
        assert not last["failures"], last["failures"]
        fin = [t for t in last["trace"] if t["quantum"] == "finish"]
        assert fin, last["trace"]
        if parallel:
            assert any(len(t.get("group") or []) == 2 for t in fin), fin
        assert last["rows"][0]["digest"]
