"""Read-only compatibility with the first archive format (schema ``...results-summary.v1``).

A v1 archive is a run directory holding ``summary.json`` with the SHA-256 of every file of the
run next to the files themselves, plus a date-stamped markdown report.  ``verify`` re-hashes
and reports missing / altered / extra files; ``inspect`` lists the summary; ``compact`` copies
the summaries and reports of every v1 run under a root and, with ``prune_raw``, deletes raw
files the summaries list.  ``finalize`` still writes this format for callers that ask for it
explicitly (``results.finalize(..., format="v1")``); the default archive is v2
(``results/__init__.py``).  Old archives grant no qualification to the current code and
cannot bring back deleted raw inputs.
Reference: workers/ditserve/results/compact.py, legacy.py (read-only compatibility).
"""
from __future__ import annotations

import datetime as _dt
import json
import shutil
from pathlib import Path

from ..runtime import file_hash

SCHEMA = "ditserve-b200.results-summary.v1"


class ResultsError(RuntimeError):
    pass


def _files(run_dir: Path):
    for p in sorted(run_dir.rglob("*")):
        if p.is_file() and p.name != "summary.json" and not p.name.endswith(".md"):
            yield p


def finalize(run_dir, title: str | None = None, date: str | None = None) -> dict:
    run = Path(run_dir)
    if not run.is_dir():
        raise ResultsError(f"{run} is not a run directory")
    files = {str(p.relative_to(run)): file_hash(p) for p in _files(run)}
    phases = {}
    for p in sorted(run.glob("phase-*.json")):
        ph = json.loads(p.read_text())
        last = ph.get("last") or {}
        phases[p.stem[len("phase-"):]] = dict(status=ph.get("status"), summary=last.get("summary"),
                                              gates=(ph.get("gates") or {}).get("pass"))
    date = date or _dt.date.today().strftime("%Y%m%d")
    summary = dict(schema=SCHEMA, run=run.name, date=date, files=files, phases=phases)
    (run / "summary.json").write_text(json.dumps(summary, indent=1, sort_keys=True))
    lines = [f"# {title or run.name}", "", f"date: {date}", "", "| phase | status | gates | SLO attainment |",
             "|---|---|---|---|"]
    for name, ph in phases.items():
        sar = (ph.get("summary") or {}).get("slo_attainment")
        lines.append(f"| {name} | {ph['status']} | {ph['gates']} | {'' if sar is None else round(sar, 4)} |")
    (run / f"{date}-{run.name}.md").write_text("\n".join(lines) + "\n")
    return summary


def verify(run_dir) -> dict:
    run = Path(run_dir)
    s = json.loads((run / "summary.json").read_text())
    if s.get("schema") != SCHEMA:
        raise ResultsError("unknown summary schema")
    present = {str(p.relative_to(run)): p for p in _files(run)}
    missing = sorted(set(s["files"]) - set(present))
    extra = sorted(set(present) - set(s["files"]))
    altered = sorted(k for k, h in s["files"].items() if k in present and file_hash(present[k]) != h)
    return dict(ok=not (missing or altered), missing=missing, altered=altered, extra=extra)


def inspect(path) -> dict:
    p = Path(path)
    s = json.loads((p / "summary.json" if p.is_dir() else p).read_text())
    return dict(run=s["run"], date=s["date"], files=len(s["files"]), phases=s["phases"])


def compact(root, destination, prune_raw: bool = False) -> dict:
    root, dest = Path(root), Path(destination)
    dest.mkdir(parents=True, exist_ok=True)
    kept, pruned = [], []
    for summary in sorted(root.rglob("summary.json")):
        run = summary.parent
        check = verify(run)
        if not check["ok"]:
            raise ResultsError(f"{run} fails verification: {check}")
        out = dest / run.name
        out.mkdir(exist_ok=True)
        shutil.copy2(summary, out / "summary.json")
        for md in run.glob("*.md"):
            shutil.copy2(md, out / md.name)
        kept.append(run.name)
        if prune_raw:
            s = json.loads(summary.read_text())
            for rel in s["files"]:
                if not rel.startswith("phase-") and rel != "run.json":
                    (run / rel).unlink(missing_ok=True)
                    pruned.append(f"{run.name}/{rel}")
    return dict(kept=kept, pruned=len(pruned))
