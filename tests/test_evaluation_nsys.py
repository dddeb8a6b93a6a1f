"""Nsight Systems SQLite parser on a synthetic export with the documented tables, and the
environment defaults of the worker runtime (packet directory, bridge endpoint)."""
import os
import sqlite3
import subprocess
import sys

import pytest

from ditserve_b200.evaluation import nsys_gpu_metrics

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _export(path):
    con = sqlite3.connect(path)
    con.executescript("""
        CREATE TABLE StringIds (id INTEGER PRIMARY KEY, value TEXT);
        CREATE TABLE CUPTI_ACTIVITY_KIND_KERNEL (start INTEGER, end INTEGER, deviceId INTEGER, streamId INTEGER,
                                                 shortName INTEGER, demangledName INTEGER);
        CREATE TABLE CUPTI_ACTIVITY_KIND_MEMCPY (start INTEGER, end INTEGER, bytes INTEGER, copyKind INTEGER,
                                                 deviceId INTEGER);
        CREATE TABLE NVTX_EVENTS (start INTEGER, end INTEGER, text TEXT);
        INSERT INTO StringIds VALUES (1, 'gemm_kernel'), (2, 'attention_kernel');
    """)
    # device 0: two overlapping kernels on two streams (busy 0..3 ms), one later (5..6 ms)
    con.executemany("INSERT INTO CUPTI_ACTIVITY_KIND_KERNEL VALUES (?,?,?,?,?,?)", [
        (0, 2_000_000, 0, 1, 1, 1), (1_000_000, 3_000_000, 0, 2, 2, 2), (5_000_000, 6_000_000, 0, 1, 2, 2),
        (0, 4_000_000, 1, 1, 1, 1)])
    con.executemany("INSERT INTO CUPTI_ACTIVITY_KIND_MEMCPY VALUES (?,?,?,?,?)", [
        (8_000_000, 9_000_000, 50_000_000, 1, 0), (9_000_000, 10_000_000, 4_000_000, 2, 0)])
    con.executemany("INSERT INTO NVTX_EVENTS VALUES (?,?,?)", [(0, 3_000_000, "step"), (3_000_000, 6_000_000, "step"),
                                                               (0, None, "open")])
    con.commit()
    con.close()


def test_nsys_metrics_from_sqlite(tmp_path):
    db = str(tmp_path / "trace.sqlite")
    _export(db)
    m = nsys_gpu_metrics(db)
    assert m["span_ms"] == pytest.approx(10.0)
    assert m["devices"][0]["busy_ms"] == pytest.approx(4.0)      # union, not the 5 ms sum
    assert m["devices"][0]["utilization"] == pytest.approx(0.4)
    assert m["devices"][1]["busy_ms"] == pytest.approx(4.0)
    names = {k["name"]: k for k in m["kernels"]}
    assert names["attention_kernel"]["calls"] == 2 and names["attention_kernel"]["total_ms"] == pytest.approx(3.0)
    assert names["gemm_kernel"]["total_ms"] == pytest.approx(6.0)
    assert m["kernels"][0]["name"] == "gemm_kernel"
    assert m["copies"]["HtoD"]["gbps"] == pytest.approx(50.0)     # 50 MB in 1 ms
    assert m["nvtx"]["step"]["count"] == 2 and "open" not in m["nvtx"]


def test_transfer_dir_environment_default(tmp_path, monkeypatch):
    from ditserve_b200.models.base import transfer_dir
    monkeypatch.setenv("DITSERVE_TRANSFER_DIR", str(tmp_path))
    assert transfer_dir({}) == str(tmp_path)
    assert transfer_dir({"transfer_dir": "/x"}) == "/x"
    monkeypatch.delenv("DITSERVE_TRANSFER_DIR")
    assert transfer_dir({}) in ("/dev/shm", "/tmp")


def test_bridge_proxy_needs_an_endpoint():
    env = {k: v for k, v in os.environ.items() if k != "DITSERVE_REMOTE_ENDPOINT"}
    env["PYTHONPATH"] = ROOT
    r = subprocess.run([sys.executable, "-m", "ditserve_b200.runtime.remote_bridge", "proxy", "--backend", "mock"],
                       capture_output=True, text=True, env=env, timeout=60)
    assert r.returncode != 0 and "DITSERVE_REMOTE_ENDPOINT" in r.stderr
