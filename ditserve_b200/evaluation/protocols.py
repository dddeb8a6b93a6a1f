"""Study generators for the reference's published serving protocols, on a measured cost profile.

    python -m ditserve_b200.evaluation.protocols modality-mix --profile configs/profiles/b200_profile.json \\
        --out configs/studies/b200_modality_mix_sim.json
    python -m ditserve_b200.evaluation.protocols reference --profile ... --out ...

Each generator writes a ``ditserve-b200.study.v1`` config whose phases the controller's simulator
(or, with real workers, the cluster executor) runs as a policy x pattern matrix:

* ``modality_mix``: 8 GPUs, 100 requests per point, deadline kappa = 1.5 x the isolated SP1
  latency including the VAE decode, video fraction v in {0.1, 0.3, 0.5, 0.7, 0.9} split evenly
  between Wan2.1 480p / Wan2.2 720p (the image share between SD3.5 512^2 / 1024^2), Poisson and
  Gamma (CV 2) arrivals, at the given arrival rates;
* ``reference_protocols``: rate scale (v 0.5, kappa 1.5, 8..36 rpm in steps of 4), SLO scale
  (12 rpm, v 0.5, kappa 1.0..2.0), the ablation staircase (76 rpm, v 0.3, kappa 1.25) and weak
  scaling (1.5 rpm per GPU on 2 / 4 / 8 / 16 GPUs with 24 / 50 / 100 / 200 requests), every rate
  multiplied by ``rate_multiplier`` so that a faster GPU sees the reference's overload factors.

Isolated latencies come from the profile: a video class costs ``steps x step_compute_ms +
decode_ms`` on one GPU, an image class its measured ``service_ms``.  The committed study configs
under ``configs/studies/`` are this module's output (``tests/test_protocols.py`` regenerates them).
Reference: the protocols of results/5.2-5.5 and benchmarks/p1_benchmark.py, formal_benchmark.py.
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path

SCHEMA = "ditserve-b200.study.v1"
VIDEO = ("wan21_480p", "wan22_720p")
IMAGE = ("sd35_512", "sd35_1024")
COMPARED = ["ditserve-b200", "ditserve", "sbp-esp-cfg2", "sbp-esp", "tetriserve", "edf-bestfit", "xdit-sp1"]
MIX_POLICIES = ["ditserve-b200", "ditserve", "ditserve-v1", "sbp-esp-cfg2", "sbp-esp", "tetriserve", "edf-bestfit",
                "edf-cfg2", "xdit-sp1"]
STAIRCASE = ["stair-base", "stair-prune", "stair-pairfit", "abl-no-cb", "ditserve", "ditserve-b200", "edf-cfg2",
             "block-cfg2"]
PATTERNS = {"axes": [{"pointer": "/generator/pattern", "values": ["poisson", "gamma"]}]}


def isolated_service_ms(profile: dict, klass: str) -> float:
    """One-GPU latency of a request of ``klass`` including its decode, from the cost profile."""
    c = profile["classes"][klass]
    if c["kind"] == "video":
        return round(c["steps"] * c["step_compute_ms"] + c["decode_ms"], 1)
    return float(c["service_ms"])


def mix_classes(profile: dict, video_fraction: float, kappa: float) -> list:
    """Generator classes: the video share split evenly between the two video classes, the rest
    between the two image classes; every deadline kappa x the isolated latency."""
    out = []
    for names, share in ((VIDEO, video_fraction), (IMAGE, 1.0 - video_fraction)):
        for klass in names:
            c = profile["classes"][klass]
            out.append(dict(weight=round(share / len(names), 10), kind=c["kind"], class_=klass,
                            service_ms=isolated_service_ms(profile, klass), slo_scale=kappa,
                            spec={"steps": c["steps"]}))
    # "class" is a keyword in Python; the JSON key is "class"
    return [{("class" if k == "class_" else k): v for k, v in c.items()} for c in out]


def _phase(pid: str, gpus: int, policies: list, profile_path: str, count: int, rate: float, classes: list,
           matrix: dict) -> dict:
    return dict(id=pid, kind="simulate", gpus=gpus, policies=list(policies), profile_path=profile_path,
                generator=dict(count=count, seed=1, pattern="poisson", rate_rpm=rate, classes=classes), matrix=matrix)


def _num(x: float):
    """Integral rates stay integers in the JSON (12, not 12.0) unless they came from a product."""
    return int(x) if float(x).is_integer() and not isinstance(x, float) else x


def modality_mix(profile: dict, profile_path: str, rates=(12, 84), fractions=(0.1, 0.3, 0.5, 0.7, 0.9),
                 gpus: int = 8, count: int = 100, kappa: float = 1.5, policies=None) -> dict:
    phases = []
    for rate in rates:
        for v in fractions:
            phases.append(_phase(f"r{rate}-v{int(round(v * 10))}", gpus, policies or MIX_POLICIES, profile_path,
                                 count, _num(rate), mix_classes(profile, v, kappa), PATTERNS))
    return dict(schema=SCHEMA, experiment="b200-modality-mix-sim",
                description=("Modality-mix protocol of the reference (8 GPUs, 100 requests per point, kappa = 1.5 x the "
                             "isolated SP1 latency incl. VAE decode, video fraction v in {0.1..0.9}, Poisson and Gamma(CV 2) "
                             "arrivals) replayed by the simulator on the measured B200 profile, at the reference's 12 rpm "
                             "and at 84 rpm (7x, the B200/A100 SP1 speed ratio, which restores the reference's load level). "
                             "Gamma uses the generator's default CV 2."),
                workers={"model": {"backend": "mock"}}, phases=phases)


def reference_protocols(profile: dict, profile_path: str, rate_multiplier: float = 7.0, count: int = 100) -> dict:
    m = rate_multiplier
    base = mix_classes(profile, 0.5, 1.5)
    phases = [
        _phase("rate-scale", 8, COMPARED, profile_path, count, 8 * m, base,
               {"axes": [{"pointer": "/generator/rate_rpm", "values": [r * m for r in range(8, 37, 4)]},
                         {"pointer": "/generator/pattern", "values": ["poisson", "gamma"]}]}),
        _phase("slo-scale", 8, COMPARED, profile_path, count, 12 * m, base,
               {"axes": [{"pointer": "/generator/classes",
                          "values": [mix_classes(profile, 0.5, k) for k in (1.0, 1.25, 1.5, 1.75, 2.0)]},
                         {"pointer": "/generator/pattern", "values": ["poisson", "gamma"]}]}),
        _phase("ablation", 8, STAIRCASE, profile_path, count, 76 * m, mix_classes(profile, 0.3, 1.25), PATTERNS),
    ]
    for g, n in ((2, 24), (4, 50), (8, 100), (16, 200)):
        phases.append(_phase(f"weak-{g}gpu", g, COMPARED, profile_path, n, 1.5 * g * m, base, PATTERNS))
    return dict(schema=SCHEMA, experiment="b200-reference-protocols-sim",
                description=("The reference's rate-scale (v 0.5, kappa 1.5, R 8-36 rpm), SLO-scale (R 12 rpm, v 0.5, "
                             "kappa 1.0-2.0) and ablation-staircase (76 rpm, v 0.3, kappa 1.25) protocols, 8 GPUs, 100 "
                             "requests per point, Poisson and Gamma(CV 2), replayed by the simulator on the measured B200 "
                             f"profile with every rate multiplied by {m:g} (the B200/A100 SP1 speed ratio of the mix) so the "
                             "load matches the reference's overload factors. Weak scaling (reference §5.5): 1.5 rpm per "
                             f"GPU x {m:g} on 2, 4, 8 and 16 GPUs with 24/50/100/200 requests, v 0.5, kappa 1.5."),
                workers={"model": {"backend": "mock"}}, phases=phases)


GENERATORS = {"modality-mix": modality_mix, "reference": reference_protocols}


def main(argv=None):
    ap = argparse.ArgumentParser(description="study configs of the reference's serving protocols")
    ap.add_argument("protocol", choices=sorted(GENERATORS))
    ap.add_argument("--profile", required=True, type=Path, help="measured cost profile (utils/calibrate.py)")
    ap.add_argument("--profile-path", default=None, help="profile path as written into the study (default: relative "
                                                         "to the output file)")
    ap.add_argument("--out", type=Path, default=None)
    args = ap.parse_args(argv)
    profile = json.loads(args.profile.read_text())
    if args.profile_path is None:
        # the study resolves profile_path against its own directory
        base = args.out.parent if args.out is not None else Path.cwd()
        profile_path = os.path.relpath(args.profile.resolve(), base.resolve())
    else:
        profile_path = args.profile_path
    study = GENERATORS[args.protocol](profile, str(profile_path))
    text = json.dumps(study, indent=1) + "\n"
    if args.out is None:
        print(text, end="")
    else:
        args.out.write_text(text)


if __name__ == "__main__":
    main()
