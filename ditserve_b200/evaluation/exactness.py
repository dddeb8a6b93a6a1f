"""Block-preemption exactness: digest comparisons on recorded runs and a live cut-schedule check.

    python -m ditserve_b200.evaluation.exactness compare --reference R --candidate C --output OUT
    python -m ditserve_b200.evaluation.exactness live [--model wan-tiny] [--device cuda] [--schedules 4]

``compare`` takes two phase records of the cluster executor (``<run>/phase-<id>.json``), one
run under a whole-step policy and one under a block-quantum policy, on the same fixed
parallel form and the same trace.  Videos are paired by their generation inputs (the request
spec minus the run-local ``request_id``), never by position.  It fails closed: a request that is
missing on one side, did not finish, has no 64-hex digest, ran under another form, or whose
arrival / deadline differ makes the comparison ``incomplete``, and so does a candidate in which no
block quantum was observed (the mechanism under test never ran) or a reference that ran one.
Reported: matched videos, digest mismatches, block quanta and held-mid-step counts, and the
paired latency deltas (p50 / p95 / p99 / max).

``live`` runs the comparison in one process on the engine itself: an uninterrupted run of a
request, then ``--schedules`` runs of the same request cut at seeded random block boundaries.
At every cut the state leaves as a continuation packet (``export_packet``) and comes back
through ``import_packet`` into a fresh request state, and some cuts also go through a
step-boundary snapshot / restore.  Every schedule must end on the uninterrupted latents
bit for bit.

Reference: benchmarks/native_exact.py:55-185 (record comparison), the reference's
fixed-form block-preemption claim; the live check has no counterpart there (the reference
only compares recorded serving runs).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import random
import re
from pathlib import Path

SCHEMA = "ditserve-b200.exactness.v1"
_HEX64 = re.compile(r"[0-9a-f]{64}")


def quantiles(values) -> dict:
    """count / p50 / p95 / p99 / max with linear interpolation between order statistics."""
    if not values:
        return dict(count=0, p50=None, p95=None, p99=None, max=None)
    xs = sorted(float(v) for v in values)

    def q(f):
        pos = (len(xs) - 1) * f
        lo = math.floor(pos)
        hi = min(lo + 1, len(xs) - 1)
        return xs[lo] + (xs[hi] - xs[lo]) * (pos - lo)
    return dict(count=len(xs), p50=q(0.5), p95=q(0.95), p99=q(0.99), max=xs[-1])


def _result(phase: dict, cell: int | None) -> dict:
    cells = phase.get("cells") or []
    if not cells:
        raise ValueError("the phase record has no cells")
    if cell is None:
        if len(cells) != 1:
            raise ValueError(f"the phase record has {len(cells)} cells; name one")
        cell = 0
    res = cells[cell].get("result")
    if not isinstance(res, dict) or "rows" not in res:
        raise ValueError("the cell has no executor result")
    return res


def _inputs_key(spec: dict) -> str:
    body = {k: v for k, v in spec.items() if k != "request_id"}
    return json.dumps(body, sort_keys=True, separators=(",", ":"))


def _quanta(res: dict) -> dict:
    """request id -> list of (form, quantum) in trace order."""
    out = {}
    for t in res.get("trace", []):
        ids = t.get("members") or [t.get("request_id")]
        for rid in ids:
            out.setdefault(rid, []).append((t.get("form"), t.get("quantum")))
    return out


def _videos(res: dict) -> dict:
    rows = {}
    for r in res["rows"]:
        if r.get("kind") != "video":
            continue
        key = _inputs_key(r.get("spec") or {})
        if key in rows:
            raise ValueError(f"two videos with the same generation inputs ({r.get('request_id')})")
        rows[key] = r
    return rows


def _block_quanta(qs) -> int:
    return sum(1 for _, q in qs if isinstance(q, (int, float)) and not isinstance(q, bool))


def compare_results(reference: dict, candidate: dict, form: str | None = None,
                    require_block_quanta: bool = True) -> dict:
    """Digest comparison of two executor results (``cells[i]["result"]`` of a phase record)."""
    ref_rows, cand_rows = _videos(reference), _videos(candidate)
    ref_q, cand_q = _quanta(reference), _quanta(candidate)
    problems, pairs, mismatches, deltas = [], [], [], []
    missing = sorted(set(ref_rows) ^ set(cand_rows))
    if missing:
        problems.append(f"{len(missing)} videos appear on one side only")
    cand_blocks = ref_blocks = 0
    for key in sorted(set(ref_rows) & set(cand_rows)):
        a, b = ref_rows[key], cand_rows[key]
        rid = b.get("request_id")
        for field in ("arrival_ms", "deadline_ms", "slo_ms"):
            if a.get(field) != b.get(field):
                problems.append(f"{rid}: {field} differs between the runs")
        digests = []
        for side, row in (("reference", a), ("candidate", b)):
            d = row.get("digest")
            if row.get("status") != "done" or not isinstance(d, str) or not _HEX64.fullmatch(d):
                problems.append(f"{row.get('request_id')}: no finished digest-bound output in the {side} run")
            digests.append(d)
        qa = [q for q in ref_q.get(a.get("request_id"), []) if q[1] != "finish"]
        qb = [q for q in cand_q.get(b.get("request_id"), []) if q[1] != "finish"]
        forms = {f for f, _ in qa + qb}
        if form is not None and forms - {form}:
            problems.append(f"{rid}: ran under {sorted(forms)}, not the controlled form {form}")
        elif form is None and len(forms) > 1:
            problems.append(f"{rid}: ran under more than one form {sorted(forms)}")
        ref_blocks += _block_quanta(qa)
        cand_blocks += _block_quanta(qb)
        pairs.append(dict(request_id=rid, reference_request_id=a.get("request_id"), reference_digest=digests[0],
                          candidate_digest=digests[1]))
        if digests[0] != digests[1]:
            mismatches.append(rid)
        if all(isinstance(r.get(k), (int, float)) for r in (a, b) for k in ("finish_ms", "arrival_ms")):
            deltas.append((b["finish_ms"] - b["arrival_ms"]) - (a["finish_ms"] - a["arrival_ms"]))
    if ref_blocks:
        problems.append(f"the whole-step reference ran {ref_blocks} block quanta")
    observed = cand_blocks > 0 or candidate.get("counters", {}).get("held_mid_step", 0) > 0
    if require_block_quanta and not observed:
        problems.append("no block quantum was observed in the candidate run")
    status = "completed" if pairs and not problems and not mismatches else "incomplete"
    return dict(schema=SCHEMA, kind="record", status=status, form=form, matched_videos=len(pairs),
                missing_identities=missing, mismatches=mismatches, problems=problems,
                candidate_block_quanta=cand_blocks,
                candidate_held_mid_step=candidate.get("counters", {}).get("held_mid_step", 0),
                mechanism_observed=observed, paired_latency_delta_ms=quantiles(deltas), pairs=pairs,
                scope="same fixed form, same trace; digest equality of the final latents")


def compare_records(reference_path, candidate_path, form=None, reference_cell=None, candidate_cell=None,
                    require_block_quanta=True) -> dict:
    raws = [Path(p).read_bytes() for p in (reference_path, candidate_path)]
    ref, cand = (json.loads(r) for r in raws)
    out = compare_results(_result(ref, reference_cell), _result(cand, candidate_cell), form, require_block_quanta)
    out["sources"] = dict(reference_sha256=hashlib.sha256(raws[0]).hexdigest(),
                          candidate_sha256=hashlib.sha256(raws[1]).hexdigest())
    return out


def cut_schedule(rng: random.Random, steps: int, layers: int, cuts: int) -> list:
    """Seeded cut points as (step, block) pairs, 0 < block < layers, sorted and distinct."""
    space = [(s, b) for s in range(steps) for b in range(1, layers)]
    return sorted(rng.sample(space, min(cuts, len(space))))


def live_check(model: str = "wan-tiny", device: str = "cuda", schedules: int = 4, cuts: int = 3, seed: int = 0,
               spec: dict | None = None) -> dict:
    """Uninterrupted run vs ``schedules`` runs cut at random block boundaries; bitwise gate."""
    import torch

    from ..models.wan.runtime import WanEngine
    spec = dict(spec or dict(model=model, height=64, width=64, frames=5, steps=3, guidance=5.0, seed=7))
    spec.setdefault("model", model)
    dev = torch.device(device)
    eng = WanEngine(spec["model"], device=dev, seed=seed)
    layers = eng.cfg.layers
    with torch.inference_mode():
        full = eng.run(eng.prepare(spec))
        want = full.latent_digest()
        rng = random.Random(seed)
        runs = []
        for k in range(schedules):
            plan = cut_schedule(rng, spec["steps"], layers, cuts)
            st = eng.prepare(spec)
            moves = []
            for step, block in plan:
                while st.step < step:                       # whole steps up to the cut's step
                    if rng.random() < 0.5 and st.block == 0:
                        st = eng.restore(eng.unpack(eng.pack(eng.snapshot(st))))
                        moves.append(["snapshot", st.step])
                    eng.advance(st)
                eng.advance(st, blocks=block - st.block)    # stop inside the step
                blob, dg = eng.export_packet(st)
                st = eng.import_packet(blob, dg)
                moves.append(["packet", st.step, st.block])
            while not st.done:
                eng.advance(st)
            got = st.latent_digest()
            runs.append(dict(schedule=[list(c) for c in plan], moves=moves, digest=got, equal=got == want))
    if dev.type == "cuda":
        from ..ops import check_status
        check_status(dev)
    ok = all(r["equal"] for r in runs)
    return dict(schema=SCHEMA, kind="live", status="completed" if ok else "mismatch", model=spec["model"],
                device=str(dev), layers=layers, spec=spec, reference_digest=want, runs=runs,
                scope="one process, one parallel form; uninterrupted vs cut at random block boundaries")


def main(argv=None):
    ap = argparse.ArgumentParser(description="block-preemption exactness")
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("compare")
    c.add_argument("--reference", required=True, type=Path)
    c.add_argument("--candidate", required=True, type=Path)
    c.add_argument("--form")
    c.add_argument("--reference-cell", type=int)
    c.add_argument("--candidate-cell", type=int)
    c.add_argument("--no-preemption", action="store_true", help="do not require observed block quanta")
    c.add_argument("--keep-pairs", action="store_true")
    c.add_argument("--output", type=Path)
    lv = sub.add_parser("live")
    lv.add_argument("--model", default="wan-tiny")
    lv.add_argument("--device", default="cuda")
    lv.add_argument("--schedules", type=int, default=4)
    lv.add_argument("--cuts", type=int, default=3)
    lv.add_argument("--seed", type=int, default=0)
    lv.add_argument("--output", type=Path)
    args = ap.parse_args(argv)
    if args.cmd == "compare":
        out = compare_records(args.reference, args.candidate, args.form, args.reference_cell, args.candidate_cell,
                              require_block_quanta=not args.no_preemption)
        if not args.keep_pairs:
            bad = set(out["mismatches"])
            out["pairs"] = [p for p in out["pairs"] if p["request_id"] in bad]
    else:
        out = live_check(args.model, args.device, args.schedules, args.cuts, args.seed)
    if args.output is not None:
        args.output.parent.mkdir(parents=True, exist_ok=True)
        with args.output.open("x") as f:
            json.dump(out, f, indent=1)
    print(json.dumps({k: out[k] for k in ("kind", "status") if k in out} |
                     {k: out[k] for k in ("matched_videos", "mismatches", "problems") if k in out} |
                     ({"runs": len(out["runs"])} if "runs" in out else {})))
    if out["status"] != "completed":
        raise SystemExit(1)


if __name__ == "__main__":
    main()
