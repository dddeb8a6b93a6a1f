"""Block-preemption exactness harness: record comparison rules and the live cut-schedule check (CPU)."""
import copy
import json

import pytest

from ditserve_b200.evaluation import exactness

D1, D2 = "a" * 64, "b" * 64


def _result(rows, trace, held=0):
    return {"rows": rows, "trace": trace, "counters": {"held_mid_step": held}}


def _row(rid, seed, digest=D1, arrival=0.0, finish=100.0):
    return {"request_id": rid, "kind": "video", "status": "done", "digest": digest, "arrival_ms": arrival,
            "deadline_ms": 500.0, "slo_ms": 500.0, "finish_ms": finish,
            "spec": {"request_id": rid, "seed": seed, "steps": 2}}


def _pair():
    ref = _result([_row("r0", 1), _row("r1", 2, D2)],
                  [{"request_id": "r0", "form": "cfg2", "quantum": "step"},
                   {"request_id": "r1", "form": "cfg2", "quantum": "step"},
                   {"request_id": "r0", "form": "cfg2", "quantum": "finish"}])
    # the candidate run names its requests differently: pairing goes by generation inputs
    cand = _result([_row("x1", 2, D2, finish=130.0), _row("x0", 1, finish=90.0)],
                   [{"request_id": "x0", "form": "cfg2", "quantum": 3},
                    {"request_id": "x0", "form": "cfg2", "quantum": "step"},
                    {"request_id": "x1", "form": "cfg2", "quantum": "step"}], held=1)
    return ref, cand


def test_compare_pairs_by_inputs_and_reports_deltas():
    ref, cand = _pair()
    out = exactness.compare_results(ref, cand, form="cfg2")
    assert out["status"] == "completed", out["problems"]
    assert out["matched_videos"] == 2 and not out["mismatches"]
    assert out["candidate_block_quanta"] == 1 and out["mechanism_observed"]
    assert out["paired_latency_delta_ms"]["count"] == 2
    assert out["paired_latency_delta_ms"]["max"] == pytest.approx(30.0)


@pytest.mark.parametrize("breakage", ["digest", "missing", "form", "no_blocks", "ref_blocks", "arrival",
                                      "unfinished"])
def test_compare_fails_closed(breakage):
    ref, cand = _pair()
    if breakage == "digest":
        cand["rows"][1]["digest"] = D2
    elif breakage == "missing":
        cand["rows"].pop(0)
    elif breakage == "form":
        cand["trace"][2]["form"] = "cfg2sp2"
    elif breakage == "no_blocks":
        cand["trace"][0]["quantum"] = "step"
        cand["counters"]["held_mid_step"] = 0
    elif breakage == "ref_blocks":
        ref["trace"][0]["quantum"] = 2
    elif breakage == "arrival":
        cand["rows"][1]["arrival_ms"] = 5.0
    elif breakage == "unfinished":
        cand["rows"][1]["status"] = "failed"
    out = exactness.compare_results(ref, cand, form="cfg2")
    assert out["status"] == "incomplete"
    if breakage == "digest":
        assert out["mismatches"] == ["x0"]
    else:
        assert out["problems"]


def test_compare_records_cli(tmp_path):
    ref, cand = _pair()
    for name, res in (("ref", ref), ("cand", cand)):
        (tmp_path / f"{name}.json").write_text(json.dumps({"cells": [{"cell": 0, "result": res}]}))
    exactness.main(["compare", "--reference", str(tmp_path / "ref.json"), "--candidate", str(tmp_path / "cand.json"),
                    "--form", "cfg2", "--output", str(tmp_path / "out.json")])
    out = json.loads((tmp_path / "out.json").read_text())
    assert out["status"] == "completed" and out["pairs"] == [] and len(out["sources"]["reference_sha256"]) == 64
    bad = copy.deepcopy(cand)
    bad["rows"][0]["digest"] = D1
    (tmp_path / "bad.json").write_text(json.dumps({"cells": [{"cell": 0, "result": bad}]}))
    with pytest.raises(SystemExit):
        exactness.main(["compare", "--reference", str(tmp_path / "ref.json"), "--candidate",
                        str(tmp_path / "bad.json")])


def test_cut_schedule_is_seeded_and_inside_steps():
    import random
    a = exactness.cut_schedule(random.Random(3), steps=4, layers=5, cuts=6)
    b = exactness.cut_schedule(random.Random(3), steps=4, layers=5, cuts=6)
    assert a == b and a == sorted(set(a)) and all(0 < blk < 5 and 0 <= s < 4 for s, blk in a)


def test_live_cut_schedules_are_bitwise_on_cpu():
    out = exactness.live_check(device="cpu", schedules=2, cuts=2, seed=1)
    assert out["status"] == "completed" and len(out["runs"]) == 2
    assert all(r["equal"] and any(m[0] == "packet" for m in r["moves"]) for r in out["runs"])
