"""Results archive: publish, verify and clean up finished study runs.

A study runs in a work directory (``<work>/<run_id>/``: ``run.json`` with the frozen config
and code identity, ``phase-<id>.json`` measurement records, worker logs and packets; the GPU
budget ledger ``budget.json`` sits one level up).  Publishing keeps two small files:

    <destination>/summary.json              schema ditserve-b200.results-summary.v2
    <destination>/YYYYMMDD-<run_id>.md      the report rendered from the summary

The summary keeps the config hash and code identity, the models served (deduplicated worker
definitions), GPU identity when the run recorded it, scalar metrics per phase, matrix cell and
modality, a qualification record, a failure digest and the cleanup receipts.  It does not copy
the full config, per-request rows, traces or time series, so a published summary cannot be
used to resume a run or to re-evaluate raw outputs.

Rules (reference: docs/results.md):
* Date: a run id that starts with YYYYMMDD- is used as is; otherwise the UTC date on which the
  run's last budget session ended; otherwise the date of the first finalize attempt (kept in
  ``<run>/.archive-date`` so a retry names the same report).
* ``finalize`` refuses without changing anything, answering ``protected`` while a budget
  session of the run is open or the ledger lock is held, and ``deferred`` while a registered
  dependency (quality evaluation, resume, re-evaluation, failure investigation) is not closed
  or while a measurement record changed since the first attempt.  A failed finalize is
  retried with the same call; an identical published summary makes it a no-op, and a
  published report is never revised by re-finalizing changed inputs (``ResultsError``).
* Qualification: ``execution`` is ``completed`` when every phase ended ok; ``numerics``,
  ``semantics`` and ``performance`` stay ``unverified`` unless a passing gate or a closed
  dependency of that kind is the evidence.  Verification of an archive only proves that the
  summary and its report agree; it grants no qualification.
* ``cleanup`` deletes only files inside the work directory that match an explicit whitelist,
  whose size and SHA-256 equal the manifest taken at finalize, and that no open dependency
  holds; a log file goes only when an aggregate bound to its hash exists
  (``<log>.aggregate.json`` with ``source_sha256``).  ``run.json``, phase records, the
  ledger and control files are never deleted.  The intent (files, hashes) is recorded before
  anything is deleted and the facts (deleted, reclaimed bytes) after.
* v1 archives (the previous format) are read through ``results.legacy``.
Reference: workers/ditserve/results/__init__.py, compact.py, legacy.py; docs/results.md.
"""
from __future__ import annotations

import datetime as _dt
import fcntl
import fnmatch
import hashlib
import json
import os
import re
from pathlib import Path

from ..runtime import file_hash
from . import legacy
from .legacy import ResultsError

SCHEMA = "ditserve-b200.results-summary.v2"
PROTECTED = ("run.json", "budget.json", "budget.json.lock", "dependencies.json", "cleanup-receipts.json",
             ".archive-date", ".finalize-intent.json", ".manifest.json")
LOG_SUFFIXES = (".log", ".err", ".out")
DEP_KINDS = ("quality", "resume", "re-evaluation", "investigation", "numerics", "semantics", "performance")
METRIC_KEYS = ("completed", "requests", "slo_attainment", "goodput_rpm", "goodput_rps", "latency_p50_ms",
               "latency_p95_ms", "latency_p99_ms", "makespan_ms", "gpu_seconds")


def _canon(obj) -> str:
    return json.dumps(obj, sort_keys=True, separators=(",", ":"))


def _sha(text: str) -> str:
    return hashlib.sha256(text.encode()).hexdigest()


def _read(p: Path):
    return json.loads(p.read_text())


def _write(p: Path, obj):
    tmp = p.with_name(p.name + ".tmp")
    tmp.write_text(json.dumps(obj, indent=1, sort_keys=True))
    os.replace(tmp, p)


# ------------------------------------------------------------------ dependencies
def _deps_path(run: Path) -> Path:
    return run / "dependencies.json"


def _deps(run: Path) -> list:
    p = _deps_path(run)
    return _read(p) if p.exists() else []


def register_dependency(run_dir, consumer: str, files, kind: str = "investigation") -> dict:
    """Record that ``consumer`` needs ``files`` (paths inside the run) until it closes."""
    run = Path(run_dir)
    if kind not in DEP_KINDS:
        raise ResultsError(f"unknown dependency kind {kind!r}")
    entries = _deps(run)
    if any(e["consumer"] == consumer and not e["closed"] for e in entries):
        raise ResultsError(f"dependency {consumer!r} is already open")
    held = {}
    for f in files:
        p = (run / f).resolve()
        if not str(p).startswith(str(run.resolve()) + os.sep) or not p.is_file():
            raise ResultsError(f"dependency file {f} is not a file of the run")
        held[str(p.relative_to(run.resolve()))] = file_hash(p)
    entry = dict(consumer=consumer, kind=kind, files=held, closed=False, result=None)
    entries.append(entry)
    _write(_deps_path(run), entries)
    return entry


def close_dependency(run_dir, consumer: str, result=None, passed: bool | None = None) -> dict:
    run = Path(run_dir)
    entries = _deps(run)
    for e in entries:
        if e["consumer"] == consumer and not e["closed"]:
            e["closed"], e["result"], e["passed"] = True, result, passed
            _write(_deps_path(run), entries)
            return e
    raise ResultsError(f"no open dependency {consumer!r}")


# ------------------------------------------------------------------ guards and dates
def _ledger(run: Path) -> Path:
    return run.parent / "budget.json"


def _open_sessions(run: Path, identity: str) -> list:
    p = _ledger(run)
    if not p.exists():
        return []
    led = _read(p)
    return [s for s in led.get("sessions", []) if s.get("state") == "open" and str(s.get("id", "")).startswith(identity)]


def _ledger_locked(run: Path) -> bool:
    lock = Path(str(_ledger(run)) + ".lock")
    if not lock.exists():
        return False
    fd = os.open(lock, os.O_RDWR)
    try:
        fcntl.flock(fd, fcntl.LOCK_EX | fcntl.LOCK_NB)
        fcntl.flock(fd, fcntl.LOCK_UN)
        return False
    except OSError:
        return True
    finally:
        os.close(fd)


def archive_date(run_dir, identity: str | None = None) -> str:
    run = Path(run_dir)
    m = re.match(r"^(\d{8})-", run.name)
    if m:
        return m.group(1)
    if identity is not None and _ledger(run).exists():
        ends = [s["end"] for s in _read(_ledger(run)).get("sessions", [])
                if str(s.get("id", "")).startswith(identity) and s.get("end") is not None]
        if ends:
            return _dt.datetime.fromtimestamp(max(ends), _dt.timezone.utc).strftime("%Y%m%d")
    p = run / ".archive-date"
    if not p.exists():
        p.write_text(_dt.datetime.now(_dt.timezone.utc).strftime("%Y%m%d"))
    return p.read_text().strip()


def _records(run: Path) -> dict:
    return {p.name: file_hash(p) for p in sorted(run.glob("phase-*.json"))}


# ------------------------------------------------------------------ summary
def _cell_metrics(cell: dict) -> dict:
    res = cell.get("result", cell)
    summ = res.get("summary") or {}
    out = {k: summ[k] for k in METRIC_KEYS if isinstance(summ.get(k), (int, float))}
    kinds = summ.get("by_kind") or summ.get("kinds") or {}
    if isinstance(kinds, dict):
        out["by_kind"] = {k: {m: v[m] for m in METRIC_KEYS if isinstance(v, dict) and isinstance(v.get(m), (int, float))}
                          for k, v in kinds.items()}
    return out


def _phase_summary(name: str, ph: dict) -> dict:
    cells = []
    for cell in ph.get("cells") or []:
        params = {k: v for k, v in (cell.get("cell") or {}).items() if isinstance(v, (int, float, str, bool))}
        cells.append(dict(params=params, metrics=_cell_metrics(cell)))
    if not cells and ph.get("last"):
        cells.append(dict(params={}, metrics=_cell_metrics(ph["last"])))
    failures = []
    for cell in ph.get("cells") or [ph.get("last") or {}]:
        res = cell.get("result", cell) if isinstance(cell, dict) else {}
        for f in res.get("failures") or []:
            failures.append(str(f)[:200])
    gates = ph.get("gates") or {}
    return dict(status=ph.get("status"), kind=ph.get("kind"), cells=cells,
                gates=dict(passed=gates.get("pass"), pointers=[g.get("pointer") for g in gates.get("results", [])
                                                               if isinstance(g, dict)]),
                failures=dict(count=len(failures), first=failures[:5]))


def _qualification(phases: dict, deps: list) -> dict:
    q = dict(execution="completed" if phases and all(p["status"] == "ok" for p in phases.values()) else "failed",
             numerics="unverified", semantics="unverified", performance="unverified")
    for p in phases.values():
        if not p["gates"]["passed"]:
            continue
        ptrs = " ".join(str(x) for x in p["gates"]["pointers"])
        if re.search(r"rel|cos|digest|psnr|ssim|lpips", ptrs):
            q["numerics"] = "verified"
        if re.search(r"slo|goodput|latency|makespan", ptrs):
            q["performance"] = "verified"
    for d in deps:
        if d["closed"] and d.get("passed") and d["kind"] in ("numerics", "semantics", "performance", "quality"):
            q["numerics" if d["kind"] == "quality" else d["kind"]] = "verified"
    return q


def _models(config: dict) -> list:
    seen, out = set(), []
    for name, w in sorted((config.get("workers") or {}).items()):
        cfg = w.get("config") or {}
        key = (w.get("backend"), cfg.get("model"), cfg.get("variant"))
        if key not in seen:
            seen.add(key)
            out.append(dict(backend=key[0], model=key[1], variant=key[2]))
    return out


def render_report(summary: dict, title: str | None = None) -> str:
    lines = [f"# {title or summary['run_id']}", "", f"date: {summary['date']}  ", f"experiment: {summary['experiment']}  ",
             f"config sha256: {summary['config_sha256'][:16]}  ", f"execution: {summary['qualification']['execution']}, "
             f"numerics: {summary['qualification']['numerics']}, performance: {summary['qualification']['performance']}",
             "", "| phase | status | gates | cell | SLO attainment | goodput (req/min) | p99 (ms) |", "|---|---|---|---|---|---|---|"]
    for name, ph in sorted(summary["phases"].items()):
        for cell in ph["cells"] or [dict(params={}, metrics={})]:
            m = cell["metrics"]
            params = ", ".join(f"{k}={v}" for k, v in sorted(cell["params"].items()))
            sar, gp, p99 = m.get("slo_attainment"), m.get("goodput_rpm"), m.get("latency_p99_ms")
            lines.append(f"| {name} | {ph['status']} | {ph['gates']['passed']} | {params} | "
                         f"{'' if sar is None else round(sar, 4)} | {'' if gp is None else round(gp, 3)} | "
                         f"{'' if p99 is None else round(p99, 1)} |")
    fails = sum(ph["failures"]["count"] for ph in summary["phases"].values())
    lines += ["", f"failures: {fails}", f"cleanup receipts: {len(summary.get('cleanup') or [])}"]
    return "\n".join(lines) + "\n"


def finalize(run_dir, destination=None, title: str | None = None, date: str | None = None, format: str = "v2") -> dict:
    """Publish a finished run (see the module docstring for the rules)."""
    if format == "v1":
        return legacy.finalize(run_dir, title, date)
    run = Path(run_dir)
    if not (run / "run.json").is_file():
        raise ResultsError(f"{run} is not a run directory (no run.json)")
    rj = _read(run / "run.json")
    identity = str(rj.get("identity", ""))
    if _open_sessions(run, identity):
        return dict(status="protected", reason="a budget session of this run is open")
    if _ledger_locked(run):
        return dict(status="protected", reason="the budget ledger is locked by a running controller")
    deps = _deps(run)
    open_deps = [d["consumer"] for d in deps if not d["closed"]]
    if open_deps:
        return dict(status="deferred", reason=f"open dependencies: {open_deps}")
    intent_p = run / ".finalize-intent.json"
    records = _records(run)
    if intent_p.exists():
        if _read(intent_p)["records"] != records:
            return dict(status="deferred", reason="measurement records changed since finalize started")
    else:
        _write(intent_p, dict(records=records))
    config = rj.get("config") or {}
    phases = {}
    for p in sorted(run.glob("phase-*.json")):
        phases[p.stem[len("phase-"):]] = _phase_summary(p.stem[len("phase-"):], _read(p))
    receipts_p = run / "cleanup-receipts.json"
    summary = dict(
        schema=SCHEMA, run_id=rj.get("run_id", run.name), experiment=config.get("experiment", ""),
        date=date or archive_date(run, identity), identity=identity, config_sha256=_sha(_canon(config)),
        source=rj.get("code") or {}, models=_models(config), gpu=rj.get("gpu"), phases=phases,
        qualification=_qualification(phases, deps), records=records,
        dependencies=[dict(consumer=d["consumer"], kind=d["kind"], passed=d.get("passed")) for d in deps],
        cleanup=_read(receipts_p) if receipts_p.exists() else [])
    report = render_report(summary, title)
    summary["report_sha256"] = _sha(report)
    dest = Path(destination) if destination is not None else run / "published"
    dest.mkdir(parents=True, exist_ok=True)
    rid = summary["run_id"]
    name = f"{rid}.md" if re.match(r"^\d{8}-", rid) else f"{summary['date']}-{rid}.md"
    sp = dest / "summary.json"
    if sp.exists():
        prev = _read(sp)
        if _canon(prev) == _canon(summary) and (dest / name).exists():
            return dict(status="finalized", resumed=True, destination=str(dest), report=name)
        raise ResultsError("a published report is never revised; publish changed inputs as a new run")
    (dest / name).write_text(report)
    _write(sp, summary)
    # manifest of the work directory at publication: what cleanup may later match against
    _write(run / ".manifest.json", {str(p.relative_to(run)): dict(sha256=file_hash(p), size=p.stat().st_size)
                                    for p in sorted(run.rglob("*")) if p.is_file() and p.name not in PROTECTED})
    return dict(status="finalized", resumed=False, destination=str(dest), report=name)


def load(path) -> dict:
    """A published summary of either format, with ``format`` set to ``v1`` or ``v2``."""
    p = Path(path)
    sp = p / "summary.json" if p.is_dir() else p
    s = _read(sp)
    if s.get("schema") == SCHEMA:
        return dict(s, format="v2")
    if s.get("schema") == legacy.SCHEMA:
        return dict(s, format="v1")
    raise ResultsError(f"unknown summary schema {s.get('schema')!r}")


def verify(path) -> dict:
    """v2: the report on disk is the one rendered from the summary (hash and content);
    v1: the run's files against their recorded hashes.  Never grants a qualification."""
    p = Path(path)
    s = load(p)
    if s["format"] == "v1":
        return dict(legacy.verify(p if p.is_dir() else p.parent), format="v1")
    d = p if p.is_dir() else p.parent
    rid = s["run_id"]
    name = f"{rid}.md" if re.match(r"^\d{8}-", rid) else f"{s['date']}-{rid}.md"
    rp = d / name
    problems = []
    if not rp.exists():
        problems.append(f"missing report {name}")
    else:
        text = rp.read_text()
        if _sha(text) != s["report_sha256"]:
            problems.append("report differs from the one recorded in the summary")
        body = {k: v for k, v in s.items() if k not in ("format", "report_sha256")}
        if render_report(body, text.splitlines()[0][2:] or None) != text:
            problems.append("report does not render from the summary")
    return dict(ok=not problems, format="v2", problems=problems, execution=s["qualification"]["execution"],
                qualification=s["qualification"])


def inspect(path) -> dict:
    s = load(path)
    if s["format"] == "v1":
        return legacy.inspect(path)
    return dict(run=s["run_id"], date=s["date"], experiment=s["experiment"], phases=sorted(s["phases"]),
                qualification=s["qualification"], models=s["models"], cleanup=len(s["cleanup"]))


def compact(root, destination, prune_raw: bool = False) -> dict:
    """Legacy (v1) compaction of every run under ``root``; v2 archives are compact already."""
    return legacy.compact(root, destination, prune_raw)


def cleanup(run_dir, whitelist, dry_run: bool = False) -> dict:
    """Delete whitelisted raw files of a published run (see the module docstring)."""
    run = Path(run_dir).resolve()
    mp = run / ".manifest.json"
    if not mp.exists():
        return dict(status="deferred", reason="the run is not published (no manifest)")
    manifest = _read(mp)
    held = {f for d in _deps(run) if not d["closed"] for f in d["files"]}
    chosen, skipped = [], []
    for p in sorted(run.rglob("*")):
        if not p.is_file():
            continue
        rel = str(p.relative_to(run))
        if not any(fnmatch.fnmatch(rel, pat) for pat in whitelist):
            continue
        why = None
        if p.name in PROTECTED or p.name.startswith("phase-") or p.name.endswith(".aggregate.json"):
            why = "protected"
        elif not str(p.resolve()).startswith(str(run) + os.sep):
            why = "outside the work directory"
        elif rel not in manifest:
            why = "not in the manifest"
        elif rel in held:
            why = "held by an open dependency"
        else:
            h = file_hash(p)
            if p.stat().st_size != manifest[rel]["size"] or h != manifest[rel]["sha256"]:
                why = "changed since publication"
            elif p.name.endswith(LOG_SUFFIXES):
                agg = p.with_name(p.name + ".aggregate.json")
                if not agg.exists() or _read(agg).get("source_sha256") != h:
                    why = "log without an aggregate bound to its hash"
        if why:
            skipped.append(dict(file=rel, reason=why))
        else:
            chosen.append(dict(file=rel, sha256=manifest[rel]["sha256"], size=manifest[rel]["size"]))
    if dry_run:
        return dict(status="dry-run", would_delete=chosen, skipped=skipped)
    receipts_p = run / "cleanup-receipts.json"
    receipts = _read(receipts_p) if receipts_p.exists() else []
    receipt = dict(intent=chosen, at=_dt.datetime.now(_dt.timezone.utc).isoformat(), deleted=[], reclaimed_bytes=0)
    receipts.append(receipt)
    _write(receipts_p, receipts)           # intent first
    for c in chosen:
        (run / c["file"]).unlink()
        receipt["deleted"].append(c["file"])
        receipt["reclaimed_bytes"] += c["size"]
    _write(receipts_p, receipts)           # then the facts
    return dict(status="cleaned", deleted=receipt["deleted"], reclaimed_bytes=receipt["reclaimed_bytes"],
                skipped=skipped)


class ResultsBackend:
    operations = ("finalize", "verify", "inspect", "compact", "cleanup", "register_dependency", "close_dependency")

    def __init__(self, config):
        self.config = config
        self.states = {}

    def capabilities(self):
        return {}

    def finalize(self, request):
        return finalize(request["path"], request.get("destination"), request.get("title"),
                        format=request.get("format", "v2"))

    def verify(self, request):
        return verify(request["path"])

    def inspect(self, request):
        return inspect(request["path"])

    def compact(self, request):
        return compact(request["path"], request["destination"], bool(request.get("prune_raw", False)))

    def cleanup(self, request):
        return cleanup(request["path"], request.get("whitelist") or [], bool(request.get("dry_run", False)))

    def register_dependency(self, request):
        return register_dependency(request["path"], request["consumer"], request.get("files") or [],
                                   request.get("kind", "investigation"))

    def close_dependency(self, request):
        return close_dependency(request["path"], request["consumer"], request.get("result"), request.get("passed"))

    def close(self):
        pass


__all__ = ["ResultsError", "ResultsBackend", "finalize", "load", "verify", "inspect", "compact", "cleanup",
           "register_dependency", "close_dependency", "archive_date", "render_report"]
