"""Prompt datasets for serving studies and quality evaluation, prepared from local files.

``prepare_dataset(kind, source, out_path, ...)`` reads one local copy of a public prompt set
(there is no download here: the caller supplies the file and, optionally, its expected SHA-256)
and writes a manifest of prompts with stable ids and a role per prompt:

* ``vbench``      ``VBench_full_info.json`` (list of {prompt_en, dimension}); every prompt kept,
                  split ``evaluation``, role ``dev`` / ``test`` for service studies;
* ``vidprom``     the VidProM CSV (``prompt`` column, optional ``uuid`` / ``time``); rows whose
                  safety scores (toxicity, obscene, identity_attack, insult, threat,
                  sexual_explicit) reach 0.5 are dropped, and a fixed-size sample is drawn by a
                  seeded hash priority in one streaming pass (the CSV never sits in memory);
* ``diffusiondb``  DiffusionDB metadata (parquet through pyarrow, or JSON lines) with a ``prompt``
                  column; NSFW-scored rows (``prompt_nsfw`` >= 0.5) are dropped, then sampled.

Roles: prompts are grouped by their normalised text so an exact duplicate can never land in
both roles; the groups are ranked by a SHA-256 of (seed, text) and the first ``dev_count``
become ``dev``, the rest ``test``.  The same file, seed and counts always give the same manifest.
Reference: workers/ditserve/evaluation/datasets.py.
"""
from __future__ import annotations

import csv
import hashlib
import heapq
import json
from pathlib import Path

SAFETY_COLUMNS = ("toxicity", "obscene", "identity_attack", "insult", "threat", "sexual_explicit")
SCHEMA = "ditserve-b200.prompt-dataset.v1"


def _h(*parts) -> str:
    return hashlib.sha256("\x1f".join(str(p) for p in parts).encode()).hexdigest()


def _file_sha(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def _norm(prompt: str) -> str:
    return " ".join(prompt.split()).lower()


def _clean(value, where) -> str:
    if not isinstance(value, str) or not value.strip():
        raise ValueError(f"empty or non-text prompt at {where}")
    return value.strip()


class _Sampler:
    """Keeps the ``n`` rows of highest seeded-hash priority seen so far (a bounded heap)."""

    def __init__(self, n: int, seed: int):
        self.n, self.seed, self.heap, self.seen = n, seed, [], 0

    def offer(self, ident: str, sample: dict):
        self.seen += 1
        pri = int(_h(self.seed, ident, sample["prompt"]), 16)
        item = (pri, self.seen, sample)
        if len(self.heap) < self.n:
            heapq.heappush(self.heap, item)
        elif item[:2] > self.heap[0][:2]:
            heapq.heapreplace(self.heap, item)

    def result(self) -> list:
        return [s for _, _, s in sorted(self.heap, key=lambda it: it[1])]  # source order


def _vbench(path: Path, _seed, _n):
    rows = json.loads(path.read_text(encoding="utf-8-sig"))
    if not isinstance(rows, list) or not rows:
        raise ValueError("VBench metadata must be a non-empty JSON list")
    out = []
    for i, row in enumerate(rows):
        row = {"prompt_en": row} if isinstance(row, str) else row
        prompt = _clean(row.get("prompt_en", row.get("prompt")), f"row {i + 1}")
        out.append(dict(sample_id=f"vbench-{i:06d}", prompt=prompt, split="evaluation",
                        dimensions=list(row.get("dimension", []))))
    return out, len(rows), 0


def _unsafe(row: dict, columns) -> bool:
    for c in columns:
        v = row.get(c)
        if v in (None, ""):
            continue
        try:
            if float(v) >= 0.5:
                return True
        except (TypeError, ValueError):
            raise ValueError(f"non-numeric safety score in column {c}")
    return False


def _vidprom(path: Path, seed, n):
    sampler, skipped = _Sampler(n, seed), 0
    with path.open(newline="", encoding="utf-8-sig") as f:
        reader = csv.DictReader(f)
        if not reader.fieldnames or "prompt" not in reader.fieldnames:
            raise ValueError("the VidProM CSV needs a prompt column")
        for i, row in enumerate(reader):
            text = row.get("prompt")
            if not isinstance(text, str) or not text.strip() or _unsafe(row, SAFETY_COLUMNS):
                skipped += 1
                continue
            ident = row.get("uuid") or row.get("id") or f"row-{i:09d}"
            sample = dict(sample_id=f"vidprom-{ident}", prompt=_clean(text, f"row {i + 2}"))
            if row.get("time"):
                sample["timestamp"] = row["time"]
            sampler.offer(ident, sample)
    if not sampler.heap:
        raise ValueError("the VidProM CSV has no usable prompt")
    return sampler.result(), sampler.seen + skipped, skipped


def _diffusiondb(path: Path, seed, n):
    sampler, skipped = _Sampler(n, seed), 0
    if path.suffix == ".parquet":
        import pyarrow.parquet as pq
        table = pq.read_table(path, columns=None)
        rows = table.to_pylist()
    else:
        rows = [json.loads(line) for line in path.read_text().splitlines() if line.strip()]
    for i, row in enumerate(rows):
        text = row.get("prompt")
        if not isinstance(text, str) or not text.strip() or _unsafe(row, ("prompt_nsfw",)):
            skipped += 1
            continue
        ident = str(row.get("image_name") or row.get("id") or f"row-{i:09d}")
        sampler.offer(ident, dict(sample_id=f"diffusiondb-{ident}", prompt=_clean(text, f"row {i + 1}")))
    if not sampler.heap:
        raise ValueError("the DiffusionDB metadata has no usable prompt")
    return sampler.result(), len(rows), skipped


READERS = {"vbench": _vbench, "vidprom": _vidprom, "diffusiondb": _diffusiondb}


def assign_roles(samples: list, dev_count: int, seed: int, key: str = "role") -> None:
    groups = sorted({_norm(s["prompt"]) for s in samples}, key=lambda t: _h(seed, t))
    if dev_count and len(groups) < 2:
        raise ValueError("at least two distinct prompts are needed for disjoint dev / test roles")
    if dev_count >= len(groups):
        raise ValueError("dev_count must leave at least one distinct test prompt")
    dev = set(groups[:dev_count])
    for s in samples:
        s[key] = "dev" if _norm(s["prompt"]) in dev else "test"


def prepare_dataset(kind: str, source, out_path=None, dev_count: int = 32, seed: int = 20261012,
                    sample_count: int = 1000, expected_sha256: str | None = None) -> dict:
    if kind not in READERS:
        raise ValueError(f"unknown dataset {kind!r}; expected one of {sorted(READERS)}")
    src = Path(source)
    if not src.is_file():
        raise LookupError(f"no local copy of {kind} at {src} (nothing is downloaded)")
    digest = _file_sha(src)
    if expected_sha256 is not None and digest != expected_sha256:
        raise ValueError(f"{src} has SHA-256 {digest[:16]}..., expected {expected_sha256[:16]}...")
    samples, rows, skipped = READERS[kind](src, seed, sample_count)
    assign_roles(samples, dev_count, seed)
    manifest = dict(schema=SCHEMA, kind=kind, source=str(src), source_sha256=digest, seed=seed, dev_count=dev_count,
                    sample_count=sample_count, rows_read=rows, rows_skipped=skipped,
                    roles={r: sum(1 for s in samples if s["role"] == r) for r in ("dev", "test")}, samples=samples)
    if out_path is not None:
        Path(out_path).write_text(json.dumps(manifest, indent=1))
    return manifest
