"""Cost-profile fitting: the Python formula matches the controller's cost model, and a fit on
measurements generated from known coefficients recovers them."""
import json
import os
import shutil
import subprocess

import pytest

from ditserve_b200.utils.fit_profile import fit, formula_ms

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "cpp", "controller", "build", "ditserve-b200")


def _profile(eff=(0.97, 0.93, 0.88), gbps=400.0, lat=0.03, overlap=0.2):
    cls = {"kind": "video", "steps": 50, "blocks_per_step": 30, "heads": 24, "step_compute_ms": 1000.0,
           "comm_mb_per_step": 40000.0, "collectives_per_step": 240, "cfg_exchange_mb": 10.0,
           "ring_mb_per_step": 8000.0}
    p = {"links": {"default_gbps": gbps, "default_latency_ms": lat}, "sp_overlap": overlap,
         "sp_efficiency": {"2": eff[0], "4": eff[1], "8": eff[2]}, "classes": {"v": cls}}
    return p


FORMS = ["sp2", "sp4", "sp8", "cfg2", "cfg2sp2", "cfg2sp4", "u2r2", "cfg2u2r2"]


@pytest.mark.skipif(not os.path.exists(BIN) or shutil.which("cmake") is None, reason="controller not built")
def test_formula_matches_controller():
    prof = _profile()
    req = {"op": "price", "profile": prof, "class": "v", "forms": FORMS}
    r = subprocess.run([BIN, "rpc", "control"], input=json.dumps(req), capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    prices = json.loads(r.stdout)
    p = dict(eff={"2": 0.97, "4": 0.93, "8": 0.88}, gbps=400.0, latency_ms=0.03, overlap=0.2)
    for f in FORMS:
        assert abs(formula_ms(prof["classes"]["v"], f, p) - prices[f]["step_ms"]) < 1e-6 * prices[f]["step_ms"], f


def test_fit_recovers_generating_coefficients():
    truth = dict(eff={"2": 0.96, "4": 0.9, "8": 0.85}, gbps=350.0, latency_ms=0.02, overlap=0.25)
    prof = _profile(eff=(0.8, 0.8, 0.8), gbps=1000.0, lat=0.1, overlap=0.0)  # poor starting values
    cls = prof["classes"]["v"]
    cls["forms"] = {f: {"step_ms": formula_ms(cls, f, truth)} for f in FORMS}
    fitted, report = fit(prof)
    assert report["rms_rel_error"] < 1e-3
    for m in report["measured"]:
        assert abs(m["formula_ms"] - m["measured_ms"]) / m["measured_ms"] < 5e-3
    assert fitted["fit"]["observations"] == len(FORMS)
