"""Study generators of the reference's serving protocols (CPU): the committed study configs are
their output on the committed B200 profile, and isolated latencies follow the profile."""
import json
import os

import pytest

from ditserve_b200.evaluation import protocols as P

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PROFILE = os.path.join(ROOT, "configs", "profiles", "b200_profile.json")


def _load(name):
    with open(os.path.join(ROOT, "configs", "studies", name)) as f:
        return json.load(f)


@pytest.mark.parametrize("name,gen", [("b200_modality_mix_sim.json", P.modality_mix),
                                      ("b200_reference_protocols_sim.json", P.reference_protocols)])
def test_committed_studies_are_generator_output(name, gen):
    with open(PROFILE) as f:
        prof = json.load(f)
    assert gen(prof, "../profiles/b200_profile.json") == _load(name)


def test_isolated_latency_and_mix_weights():
    prof = {"classes": {
        "wan21_480p": {"kind": "video", "steps": 50, "step_compute_ms": 500.0, "decode_ms": 1000.0},
        "wan22_720p": {"kind": "video", "steps": 40, "step_compute_ms": 1000.0, "decode_ms": 3000.0},
        "sd35_512": {"kind": "image", "steps": 28, "service_ms": 400.0},
        "sd35_1024": {"kind": "image", "steps": 28, "service_ms": 1100.0}}}
    assert P.isolated_service_ms(prof, "wan21_480p") == 26000.0
    assert P.isolated_service_ms(prof, "sd35_1024") == 1100.0
    cls = P.mix_classes(prof, 0.3, 1.25)
    assert [c["class"] for c in cls] == ["wan21_480p", "wan22_720p", "sd35_512", "sd35_1024"]
    assert [c["weight"] for c in cls] == [0.15, 0.15, 0.35, 0.35]
    assert all(c["slo_scale"] == 1.25 for c in cls) and cls[1]["spec"] == {"steps": 40}
    ref = P.reference_protocols(prof, "p.json", rate_multiplier=2)
    ids = [p["id"] for p in ref["phases"]]
    assert ids == ["rate-scale", "slo-scale", "ablation", "weak-2gpu", "weak-4gpu", "weak-8gpu", "weak-16gpu"]
    assert ref["phases"][0]["matrix"]["axes"][0]["values"] == [16, 24, 32, 40, 48, 56, 64, 72]
    assert ref["phases"][2]["generator"]["rate_rpm"] == 152
    assert [p["generator"]["rate_rpm"] for p in ref["phases"][3:]] == [6.0, 12.0, 24.0, 48.0]


def test_cli_writes_a_study_with_a_relative_profile_path(tmp_path):
    out = tmp_path / "mix.json"
    P.main(["modality-mix", "--profile", PROFILE, "--out", str(out)])
    study = json.loads(out.read_text())
    assert study["schema"] == P.SCHEMA and len(study["phases"]) == 10
    path = study["phases"][0]["profile_path"]
    assert not os.path.isabs(path) and os.path.samefile(os.path.join(tmp_path, path), PROFILE)
