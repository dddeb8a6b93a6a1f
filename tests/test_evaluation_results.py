"""Quality metrics, dataset splits, trace parsing and the results archive (CPU)."""
import json

import pytest
import torch

from ditserve_b200.evaluation import drift, hash_bucket_split, kineto_summary, lpips, psnr, ssim
from ditserve_b200.results import ResultsError, compact, finalize, inspect, verify


def test_quality_metrics():
    a = torch.rand(1, 3, 4, 32, 32) * 2 - 1
    assert psnr(a, a) == float("inf") and abs(ssim(a, a) - 1) < 1e-5
    b = (a + 0.1 * torch.randn_like(a)).clamp(-1, 1)
    assert 15 < psnr(a, b) < 40 and ssim(a, b) < 0.99
    d = drift(a, b)
    assert d["passes"] and d["cos"] > 0.95
    with pytest.raises(RuntimeError):
        lpips(a, b)


def test_hash_bucket_split_is_stable():
    ids = [f"prompt-{i}" for i in range(1000)]
    s1, s2 = hash_bucket_split(ids), hash_bucket_split(list(reversed(ids)))
    assert {k: sorted(v) for k, v in s1.items()} == {k: sorted(v) for k, v in s2.items()}
    assert 700 < len(s1["train"]) < 900


def test_kineto_summary(tmp_path):
    trace = {"traceEvents": [{"ph": "X", "cat": "kernel", "name": "gemm", "dur": 30},
                             {"ph": "X", "cat": "kernel", "name": "attn", "dur": 70},
                             {"ph": "X", "cat": "cpu_op", "name": "aten::mm", "dur": 5}]}
    p = tmp_path / "t.json"
    p.write_text(json.dumps(trace))
    rows = kineto_summary(str(p))
    assert rows[0]["name"] == "attn" and rows[0]["share"] == 0.7


def test_results_archive(tmp_path):
    run = tmp_path / "runs" / "r1"
    run.mkdir(parents=True)
    (run / "phase-a.json").write_text(json.dumps({"status": "ok", "last": {"summary": {"slo_attainment": 0.9}},
                                                  "gates": {"pass": True}}))
    (run / "raw.bin").write_bytes(b"\x00" * 10)
    s = finalize(run, date="20261201", format="v1")  # the previous archive format, still writable
    assert s["phases"]["a"]["summary"]["slo_attainment"] == 0.9
    assert (run / "20261201-r1.md").exists()
    assert verify(run)["ok"] and verify(run)["format"] == "v1" and inspect(run)["files"] == 2
    (run / "raw.bin").write_bytes(b"\x01" * 10)
    assert verify(run)["altered"] == ["raw.bin"]
    with pytest.raises(ResultsError):
        compact(tmp_path / "runs", tmp_path / "archive")
    (run / "raw.bin").write_bytes(b"\x00" * 10)
    out = compact(tmp_path / "runs", tmp_path / "archive", prune_raw=True)
    assert out["kept"] == ["r1"] and not (run / "raw.bin").exists()
    assert (tmp_path / "archive" / "r1" / "summary.json").exists()
