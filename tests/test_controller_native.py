"""The C++ controller: ctest suites and an end-to-end CPU study through the CLI."""
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
    subprocess.run(["cmake", "-S", CTL, "-B", BUILD, "-DCMAKE_BUILD_TYPE=Release"], check=True,
                   capture_output=True)
    subprocess.run(["cmake", "--build", BUILD, "-j", str(os.cpu_count() or 4)], check=True, capture_output=True)
    return BIN


def test_ctest_suites(controller):
    r = subprocess.run(["ctest", "--output-on-failure"], cwd=BUILD, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def test_rpc_needs_no_python(controller):
    req = {"state": {"now_ms": 0, "gpus": 8, "requests": [
        {"request_id": "v", "kind": "video", "class": "wan21_480p", "arrival_ms": 0, "deadline_ms": 1e9}]},
           "policy": "ditserve"}
    r = subprocess.run([controller, "rpc", "plan"], input=json.dumps(req), capture_output=True, text=True,
                       env={"PATH": "/usr/bin:/bin"})
    assert r.returncode == 0, r.stderr
    plan = json.loads(r.stdout)
    assert plan["assignments"][0]["request_id"] == "v"
    cat = json.loads(subprocess.run([controller, "rpc", "policies"], input="{}", capture_output=True,
                                    text=True).stdout)
    assert {"ditserve", "tetriserve", "edf-bestfit"} <= {p["id"] for p in cat}
    bad = subprocess.run([controller, "rpc", "nope"], input="{}", capture_output=True, text=True)
    assert bad.returncode == 2


def test_mock_study_end_to_end(controller, tmp_path):
    env = dict(os.environ, DITSERVE_PYTHON=sys.executable, DITSERVE_PACKAGE_ROOT=ROOT)
    cfg = os.path.join(ROOT, "configs", "studies", "mock.json")
    r = subprocess.run([controller, "--json", "run", "--config", cfg, "--run-id", "t1", "--work-dir", str(tmp_path)],
                       capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    rep = json.loads(r.stdout)
    assert rep["status"] == "ok"
    for pid in ("online", "online-arms", "cluster"):
        assert rep["phases"][pid]["gates"]["pass"], rep["phases"][pid]["gates"]
    sims = rep["phases"]["whatif"]["last"]
    assert set(sims) == {"ditserve", "edf-bestfit", "static-cfg2sp4", "xdit-sp1"}
    # resume refuses a changed config and skips finished phases otherwise
    again = subprocess.run([controller, "--json", "run", "--config", cfg, "--run-id", "t1", "--work-dir",
                            str(tmp_path), "--resume"], capture_output=True, text=True, env=env, timeout=600)
    assert again.returncode == 0 and json.loads(again.stdout)["phases"]["ops"]["resumed"]
    no = subprocess.run([controller, "run", "--config", cfg, "--run-id", "t1", "--work-dir", str(tmp_path)],
                        capture_output=True, text=True, env=env)
    assert no.returncode == 1


def test_results_cli(controller, tmp_path):
    """results finalize publishes a v2 summary + report, verify checks it, cleanup removes a
    whitelisted raw file only after publication, and the v1 format stays writable and readable."""
    run = tmp_path / "work" / "r1"
    run.mkdir(parents=True)
    (run / "run.json").write_text(json.dumps({"run_id": "r1", "identity": "abc", "config": {"experiment": "e"},
                                              "code": {}}))
    (run / "phase-a.json").write_text(json.dumps({"status": "ok", "last": {"summary": {"slo_attainment": 1.0}},
                                                  "gates": {"pass": True}}))
    (run / "raw.bin").write_bytes(b"\x00" * 8)
    env = dict(os.environ, DITSERVE_PYTHON=sys.executable, DITSERVE_PACKAGE_ROOT=ROOT)

    def cli(*args):
        return subprocess.run([controller, "--json", "results", *args], capture_output=True, text=True, env=env,
                              timeout=300)
    dest = tmp_path / "published"
    fin = cli("finalize", str(run), "--output", str(dest), "--title", "t")
    assert fin.returncode == 0, fin.stderr
    assert json.loads(fin.stdout)["status"] == "finalized"
    ver = cli("verify", str(dest))
    assert ver.returncode == 0 and json.loads(ver.stdout)["ok"]
    dry = cli("cleanup", str(run), "--whitelist", "*.bin", "--dry-run")
    assert [c["file"] for c in json.loads(dry.stdout)["would_delete"]] == ["raw.bin"]
    out = cli("cleanup", str(run), "--whitelist", "*.bin")
    assert json.loads(out.stdout)["reclaimed_bytes"] == 8 and not (run / "raw.bin").exists()
    old = tmp_path / "old"
    old.mkdir()
    (old / "phase-a.json").write_text(json.dumps({"status": "ok"}))
    assert cli("finalize", str(old), "--v1").returncode == 0
    assert json.loads(cli("verify", str(old)).stdout)["format"] == "v1"
    bad = subprocess.run([controller, "results", "explode", str(run)], capture_output=True, text=True, env=env)
    assert bad.returncode == 2


def test_resume_refuses_changed_worker_sources(controller, tmp_path):
    """run.json freezes the controller binary and worker package hashes; a changed source file
    makes --resume refuse."""
    pkg = tmp_path / "pkgroot"
    shutil.copytree(os.path.join(ROOT, "ditserve_b200"), pkg / "ditserve_b200",
                    ignore=shutil.ignore_patterns("__pycache__", "*.so"))
    cfg = {"schema": "ditserve-b200.study.v1", "experiment": "freeze",
           "workers": {"model": {"backend": "mock"}},
           "phases": [{"id": "ops", "kind": "operations", "operations": [
               {"op": "prepare", "spec": {"request_id": "a", "steps": 1, "seed": 1}}]}]}
    cfgp = tmp_path / "s.json"
    cfgp.write_text(json.dumps(cfg))
    env = dict(os.environ, DITSERVE_PYTHON=sys.executable, DITSERVE_PACKAGE_ROOT=str(pkg))
    cmd = [controller, "--json", "run", "--config", str(cfgp), "--run-id", "f", "--work-dir", str(tmp_path / "w")]
    first = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=300)
    assert first.returncode == 0, first.stderr
    assert json.loads(first.stdout)["code"]["files"] > 10
    same = subprocess.run(cmd + ["--resume"], capture_output=True, text=True, env=env, timeout=300)
    assert same.returncode == 0, same.stderr
    with open(pkg / "ditserve_b200" / "models" / "mock.py", "a") as f:
        f.write("\n# edited\n")
    changed = subprocess.run(cmd + ["--resume"], capture_output=True, text=True, env=env, timeout=300)
    assert changed.returncode != 0 and "refusing to resume" in (changed.stdout + changed.stderr)


def test_operations_phase_on_a_remote_worker(controller, tmp_path):
    """A worker definition with "remote": "host:port" runs behind the bridge proxy in any phase."""
    env = dict(os.environ, PYTHONPATH=ROOT, DITSERVE_BRIDGE_TOKEN="t0k")
    d = subprocess.Popen([sys.executable, "-m", "ditserve_b200.runtime.remote_bridge", "daemon", "--listen",
                          "127.0.0.1:0"], stdout=subprocess.PIPE, text=True, env=env, cwd=str(tmp_path))
    try:
        port = json.loads(d.stdout.readline())["listening"]
        cfg = {"schema": "ditserve-b200.study.v1", "experiment": "remote-ops",
               "workers": {"model": {"backend": "mock", "remote": f"127.0.0.1:{port}"}},
               "phases": [{"id": "ops", "kind": "operations", "operations": [
                   {"op": "prepare", "spec": {"request_id": "a", "steps": 2, "seed": 1}},
                   {"op": "advance", "state_id": "a", "steps": 2},
                   {"op": "finish", "state_id": "a", "output_mode": "digest"}]}]}
        cfgp = tmp_path / "s.json"
        cfgp.write_text(json.dumps(cfg))
        run_env = dict(os.environ, DITSERVE_PYTHON=sys.executable, DITSERVE_PACKAGE_ROOT=ROOT,
                       DITSERVE_BRIDGE_TOKEN="t0k")
        r = subprocess.run([controller, "--json", "run", "--config", str(cfgp), "--run-id", "r", "--work-dir",
                            str(tmp_path / "w")], capture_output=True, text=True, env=run_env, timeout=300)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
        rows = json.loads(r.stdout)["phases"]["ops"]["cells"][-1]["result"]["operations"]
        assert all(x["ok"] for x in rows) and rows[-1]["result"]["value"]
    finally:
        d.terminate()
        d.wait(timeout=10)
