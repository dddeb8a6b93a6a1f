"""Results archive v2: publication rules, dependency closure, guarded cleanup and the v1 reader."""
import fcntl
import json
import os

import pytest

from ditserve_b200.results import (ResultsError, archive_date, cleanup, close_dependency, finalize, inspect, load,
                                   register_dependency, verify)


def _run(tmp_path, run_id="mix-abc123", status="ok", gates_pass=True):
    work = tmp_path / "work"
    run = work / run_id
    run.mkdir(parents=True)
    config = {"experiment": "mix", "workers": {"wan": {"backend": "wan", "config": {"model": "wan2.1-t2v-1.3b"}},
                                               "wan_b": {"backend": "wan", "config": {"model": "wan2.1-t2v-1.3b"}},
                                               "img": {"backend": "sd35", "config": {"model": "sd3.5-medium"}}}}
    (run / "run.json").write_text(json.dumps({"run_id": run_id, "identity": "id42", "config": config,
                                              "code": {"controller": "c0ffee", "worker": "beef"}}))
    phase = {"status": status, "kind": "cluster", "gates": {"pass": gates_pass,
                                                             "results": [{"pointer": "/last/summary/slo_attainment"}]},
             "cells": [{"cell": {"policy": "ditserve", "rate_rpm": 2},
                        "result": {"summary": {"slo_attainment": 0.91, "goodput_rpm": 1.8, "latency_p99_ms": 41000.0,
                                               "completed": 40, "by_kind": {"video": {"slo_attainment": 0.88}}},
                                   "failures": []}},
                       {"cell": {"policy": "edf-bestfit", "rate_rpm": 2},
                        "result": {"summary": {"slo_attainment": 0.75, "completed": 40},
                                   "failures": ["worker 3 exited"]}}]}
    (run / "phase-online.json").write_text(json.dumps(phase))
    (run / "worker-0.log").write_text("step 1\nstep 2\n")
    (run / "packet-1.bin").write_bytes(b"\x01" * 64)
    (run / "packet-2.bin").write_bytes(b"\x02" * 64)
    ledger = {"sessions": [{"id": "id42/online", "start": 1764600000.0, "end": 1764631000.0, "state": "settled"}]}
    (work / "budget.json").write_text(json.dumps(ledger))
    return run


def test_publish_summary_and_report(tmp_path):
    run = _run(tmp_path)
    dest = tmp_path / "results" / "mix" / "run1"
    out = finalize(run, dest)
    assert out["status"] == "finalized" and not out["resumed"]
    s = load(dest)
    assert s["format"] == "v2" and s["date"] == "20251201"           # the ledger's last session end (UTC)
    assert out["report"] == "20251201-mix-abc123.md" and (dest / out["report"]).exists()
    assert s["models"] == [{"backend": "sd35", "model": "sd3.5-medium", "variant": None},
                           {"backend": "wan", "model": "wan2.1-t2v-1.3b", "variant": None}]
    cells = s["phases"]["online"]["cells"]
    assert cells[0]["metrics"]["slo_attainment"] == 0.91 and cells[0]["params"]["policy"] == "ditserve"
    assert cells[0]["metrics"]["by_kind"]["video"]["slo_attainment"] == 0.88
    assert s["phases"]["online"]["failures"]["count"] == 1
    assert s["qualification"] == {"execution": "completed", "numerics": "unverified", "semantics": "unverified",
                                  "performance": "verified"}
    assert "config" not in s and "rows" not in json.dumps(s)        # no full config, no per-request rows
    assert verify(dest)["ok"]
    # a retry is a no-op; tampering with the report is caught; revising is refused
    assert finalize(run, dest)["resumed"]
    rp = dest / out["report"]
    rp.write_text(rp.read_text() + "edited\n")
    assert not verify(dest)["ok"]
    rp.write_text(rp.read_text().replace("edited\n", ""))
    assert verify(dest)["ok"]
    ph = json.loads((run / "phase-online.json").read_text())
    ph["cells"][0]["result"]["summary"]["slo_attainment"] = 0.99
    (run / "phase-online.json").write_text(json.dumps(ph))
    assert finalize(run, dest)["status"] == "deferred"              # a measurement record changed


def test_dates():
    from pathlib import Path
    assert archive_date(Path("/nonexistent/20260105-x")) == "20260105"


def test_report_name_keeps_a_dated_run_id(tmp_path):
    run = _run(tmp_path, run_id="20260102-abc")
    out = finalize(run, tmp_path / "dest")
    assert out["report"] == "20260102-abc.md" and load(tmp_path / "dest")["date"] == "20260102"


def test_guards_protect_open_sessions_locks_and_dependencies(tmp_path):
    run = _run(tmp_path)
    ledger = run.parent / "budget.json"
    led = json.loads(ledger.read_text())
    led["sessions"].append({"id": "id42/online", "start": 1.0, "end": None, "state": "open"})
    ledger.write_text(json.dumps(led))
    assert finalize(run, tmp_path / "d")["status"] == "protected"
    led["sessions"].pop()
    ledger.write_text(json.dumps(led))
    lock = open(str(ledger) + ".lock", "w")
    fcntl.flock(lock, fcntl.LOCK_EX)
    try:
        import subprocess
        import sys
        code = ("import sys;from ditserve_b200.results import finalize;"
                f"print(finalize({str(run)!r}, {str(tmp_path / 'd')!r})['status'])")
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120,
                           env=dict(os.environ, PYTHONPATH=os.getcwd()))
        assert r.stdout.strip() == "protected", r.stdout + r.stderr
    finally:
        fcntl.flock(lock, fcntl.LOCK_UN)
        lock.close()
    register_dependency(run, "vbench", ["packet-1.bin"], kind="quality")
    assert finalize(run, tmp_path / "d")["status"] == "deferred"
    with pytest.raises(ResultsError):
        register_dependency(run, "vbench", ["packet-1.bin"], kind="quality")
    with pytest.raises(ResultsError):
        register_dependency(run, "x", ["../budget.json"])
    close_dependency(run, "vbench", result={"score": 0.8}, passed=True)
    out = finalize(run, tmp_path / "d")
    assert out["status"] == "finalized"
    assert load(tmp_path / "d")["qualification"]["numerics"] == "verified"   # a passed quality evaluation


def test_cleanup_is_whitelisted_hash_checked_and_receipted(tmp_path):
    run = _run(tmp_path)
    assert cleanup(run, ["*.bin"])["status"] == "deferred"            # not published yet
    finalize(run, tmp_path / "d")
    register_dependency(run, "replay", ["packet-2.bin"], kind="resume")
    (run / "late.bin").write_bytes(b"\x03")                             # not in the manifest
    dry = cleanup(run, ["*.bin", "*.log", "run.json", "phase-*"], dry_run=True)
    assert [c["file"] for c in dry["would_delete"]] == ["packet-1.bin"]
    reasons = {s["file"]: s["reason"] for s in dry["skipped"]}
    assert reasons["packet-2.bin"] == "held by an open dependency"
    assert reasons["late.bin"] == "not in the manifest"
    assert reasons["worker-0.log"] == "log without an aggregate bound to its hash"
    assert reasons["run.json"] == "protected" and reasons["phase-online.json"] == "protected"
    from ditserve_b200.runtime import file_hash
    (run / "worker-0.log.aggregate.json").write_text(json.dumps({"source_sha256": file_hash(run / "worker-0.log"),
                                                                 "lines": 2}))
    out = cleanup(run, ["*.bin", "*.log"])
    assert sorted(out["deleted"]) == ["packet-1.bin", "worker-0.log"] and out["reclaimed_bytes"] == 64 + 14
    receipts = json.loads((run / "cleanup-receipts.json").read_text())
    assert receipts[-1]["intent"] and receipts[-1]["deleted"]
    assert (run / "run.json").exists() and (run / "packet-2.bin").exists()


def test_v1_archives_are_read(tmp_path):
    from ditserve_b200.results import legacy
    run = tmp_path / "old"
    run.mkdir()
    (run / "phase-a.json").write_text(json.dumps({"status": "ok", "last": {"summary": {"slo_attainment": 0.5}}}))
    legacy.finalize(run, date="20250101")
    assert load(run)["format"] == "v1"
    assert verify(run)["ok"] and verify(run)["format"] == "v1"
    assert inspect(run)["date"] == "20250101"
