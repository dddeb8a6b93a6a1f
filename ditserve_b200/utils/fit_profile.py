"""Fit the analytical cost model's shared coefficients to a profile's measured forms.

    python -m ditserve_b200.utils.fit_profile --profile configs/profiles/b200_profile.json --out fitted.json

The planner prices a video form from the class's single-GPU compute time plus communication:

    step = compute / (cfg * sp * eff(sp)) + comm_mb / cfg * (u - 1) / u^2 / gbps * (u / sp)
           + collectives / cfg * latency_ms + [cfg = 2] (cfg_exchange_mb / gbps + latency_ms)
           + ring term - [cfg = 1, sp > 1] overlap * min(compute term, comm term)

(u = Ulysses degree).  Measured forms (``classes.<c>.forms.<form>.step_ms``) override the formula
for themselves; every other form comes from the formula, so its coefficients decide how well the
planner prices the forms that were not measured.  This fits the shared coefficients — the SP
efficiency per degree, the link rate and latency, the SP overlap — by least squares on the relative
error of every measured multi-GPU form of every video class, then reports the residuals and the
formula's price of each form next to its measurement.  Reference: the native-profile fitting of
the reference's benchmark tooling (benchmarks/fit_native_profile.py).
"""
from __future__ import annotations

import argparse
import json
import math

import numpy as np


def parse_form(name: str) -> tuple[int, int, int]:
    """'sp4' -> (1, 4, 1); 'cfg2sp2' -> (2, 2, 1); 'u2r2' -> (1, 4, 2); 'cfg2' -> (2, 1, 1)."""
    cfg, rest = (2, name[4:]) if name.startswith("cfg2") else (1, name)
    if not rest:
        return cfg, 1, 1
    if rest.startswith("sp"):
        return cfg, int(rest[2:]), 1
    if rest.startswith("u"):
        u, r = rest[1:].split("r")
        return cfg, int(u) * int(r), int(r)
    raise ValueError(f"bad form {name!r}")


def formula_ms(cls: dict, form: str, p: dict) -> float:
    cfg, sp, ring = parse_form(form)
    eff = 1.0 if sp == 1 else p["eff"].get(str(sp), 1.0)
    compute = cls["step_compute_ms"] / (cfg * sp * eff)
    comm = lat = ring_t = exch = overlap = 0.0
    if sp > 1:
        u = sp // ring
        comm = cls.get("comm_mb_per_step", 0.0) / cfg * (u - 1) / (u * u) / p["gbps"] * (u / sp)
        lat = cls.get("collectives_per_step", 0.0) / cfg * p["latency_ms"]
    if ring > 1:
        ring_t = cls.get("ring_mb_per_step", 0.0) / cfg * (ring - 1) / (sp * ring) / p["gbps"]
    if cfg == 2:
        exch = cls.get("cfg_exchange_mb", 0.0) / p["gbps"] + p["latency_ms"]
    if cfg == 1 and sp > 1:
        overlap = p["overlap"] * min(compute, comm)
    return compute + comm + lat + ring_t + exch - overlap


def _observations(profile: dict):
    obs = []
    for name, cls in profile["classes"].items():
        if cls.get("kind") != "video" or not cls.get("step_compute_ms"):
            continue
        for form, m in (cls.get("forms") or {}).items():
            if parse_form(form) != (1, 1, 1) and "step_ms" in m:
                obs.append((name, form, float(m["step_ms"])))
    return obs


def fit(profile: dict, degrees=(2, 4, 8)) -> tuple[dict, dict]:
    """Returns (fitted profile, report)."""
    from scipy.optimize import least_squares
    obs = _observations(profile)
    if not obs:
        raise ValueError("no measured multi-GPU forms to fit")
    links = profile.get("links", {})
    eff0 = profile.get("sp_efficiency", {})
    x0 = [float(eff0.get(str(d), 0.95)) if isinstance(eff0, dict) else 0.95 for d in degrees]
    x0 += [float(links.get("default_gbps", 700.0)), float(links.get("default_latency_ms", 0.02)),
           float(profile.get("sp_overlap", 0.0))]
    lo = [0.3] * len(degrees) + [10.0, 1e-4, 0.0]
    hi = [1.0] * len(degrees) + [5000.0, 5.0, 1.0]  # no super-linear SP efficiency

    def unpack(x):
        return dict(eff={str(d): x[i] for i, d in enumerate(degrees)}, gbps=x[len(degrees)],
                    latency_ms=x[len(degrees) + 1], overlap=x[len(degrees) + 2])

    def residuals(x):
        p = unpack(x)
        return np.array([(formula_ms(profile["classes"][c], f, p) - m) / m for c, f, m in obs])

    x0 = np.clip(np.array(x0), lo, hi)
    res = least_squares(residuals, x0, bounds=(lo, hi))
    p = unpack(res.x)
    out = json.loads(json.dumps(profile))
    out["sp_efficiency"] = {k: round(v, 4) for k, v in p["eff"].items()}
    out.setdefault("links", {})["default_gbps"] = round(p["gbps"], 2)
    out["links"]["default_latency_ms"] = round(p["latency_ms"], 5)
    out["sp_overlap"] = round(p["overlap"], 4)
    report = dict(parameters=dict(sp_efficiency=out["sp_efficiency"], gbps=out["links"]["default_gbps"],
                                  latency_ms=out["links"]["default_latency_ms"], sp_overlap=out["sp_overlap"]),
                  rms_rel_error=float(math.sqrt(np.mean(res.fun ** 2))), measured=[], predicted={})
    for c, f, m in obs:
        report["measured"].append(dict(klass=c, form=f, measured_ms=m,
                                       formula_ms=round(formula_ms(out["classes"][c], f, p), 2)))
    for c, cls in out["classes"].items():
        if cls.get("kind") != "video" or not cls.get("step_compute_ms"):
            continue
        heads = cls.get("heads", 0)
        for form in ("sp2", "sp4", "sp8", "cfg2", "cfg2sp2", "cfg2sp4", "u2r2", "cfg2u2r2"):
            cfg, sp, ring = parse_form(form)
            if heads and heads % (sp // ring):
                continue
            report["predicted"].setdefault(c, {})[form] = round(formula_ms(cls, form, p), 2)
    out["fit"] = dict(rms_rel_error=round(report["rms_rel_error"], 5), observations=len(obs))
    return out, report


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--profile", required=True)
    ap.add_argument("--out", required=True)
    args = ap.parse_args(argv)
    fitted, report = fit(json.load(open(args.profile)))
    json.dump(fitted, open(args.out, "w"), indent=1)
    print(json.dumps(report, indent=1))


if __name__ == "__main__":
    main()
