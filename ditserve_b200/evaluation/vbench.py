"""VBench quality evaluation against one pinned official checkout.

Three steps, each refusing rather than guessing:

1. ``generation_protocol(full_info_path, dimensions)`` turns the official ``VBench_full_info.json``
   of the pinned checkout into the list of videos to generate: every (dimension, prompt) pair
   of the requested dimensions with five seeds (25 for ``temporal_flickering``), a file name per
   video, and a SHA-256 seal over the canonical content.  No video or weight is fetched.
2. ``export_videos(videos, protocol, videos_dir)`` writes the generated videos (uint8 or [-1, 1]
   tensors [3, T, H, W]) under the protocol's names with ffmpeg; a missing ffmpeg, a missing
   or duplicate (prompt, seed), or a shape that differs from the protocol's generation settings
   is an error, and an existing file is only accepted when its hash matches the record.
3. ``run_vbench(protocol_path, videos_dir, repo_dir)`` checks that ``repo_dir`` is a clean
   checkout at ``VBENCH_REVISION`` and that the protocol and the video set are unchanged, then
   runs the official ``evaluate.py`` per dimension under one deadline and collects its scores.
   Any mismatch (revision, dirty tree, altered protocol, missing or changed video, failing or
   incomplete evaluator output) raises; there is no partial score.

The pinned tool (repository, commit, version) and the seed counts are VBench's protocol, kept
as VBench defines them.  Reference: workers/ditserve/evaluation/vbench.py.
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import subprocess
import sys
import time
from pathlib import Path

VBENCH_REPOSITORY = "https://github.com/Vchitect/VBench"
VBENCH_REVISION = "1039fe66d7aa2f4b214003ca2d35f5011c48bfee"
VBENCH_VERSION = "v0.1.5"
DIMENSIONS = ("subject_consistency", "background_consistency", "temporal_flickering", "motion_smoothness",
              "dynamic_degree", "aesthetic_quality", "imaging_quality", "object_class", "multiple_objects",
              "human_action", "color", "spatial_relationship", "scene", "temporal_style", "appearance_style",
              "overall_consistency")
PROTOCOL_SCHEMA = "ditserve-b200.vbench-protocol.v1"


def _sha_file(path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def _seal(obj: dict) -> dict:
    body = {k: v for k, v in obj.items() if k != "seal"}
    return dict(body, seal=hashlib.sha256(json.dumps(body, sort_keys=True, separators=(",", ":")).encode()).hexdigest())


def _sealed(obj: dict) -> bool:
    return obj.get("seal") == _seal(obj)["seal"]


def _seeds(dimension: str) -> int:
    return 25 if dimension == "temporal_flickering" else 5


def generation_protocol(full_info_path, dimensions=None, settings: dict | None = None) -> dict:
    src = Path(full_info_path)
    info = json.loads(src.read_text())
    dims = list(dimensions or DIMENSIONS)
    if not dims or len(set(dims)) != len(dims) or set(dims) - set(DIMENSIONS):
        raise ValueError(f"invalid VBench dimensions {dims}")
    if not isinstance(info, list) or not info:
        raise ValueError("VBench_full_info must be a non-empty list")
    videos, seen = [], set()
    for entry in info:
        prompt = entry.get("prompt_en")
        if not isinstance(prompt, str) or not prompt or any(c in prompt for c in "/\\\0"):
            raise ValueError(f"unusable prompt as a file name: {prompt!r}")
        for dim in entry.get("dimension", []):
            if dim not in dims:
                continue
            if (dim, prompt) in seen:
                raise ValueError(f"duplicate prompt {prompt!r} in {dim}")
            seen.add((dim, prompt))
            videos += [dict(dimension=dim, prompt=prompt, seed=s, path=f"{dim}/{prompt}-{s}.mp4")
                       for s in range(_seeds(dim))]
    missing = set(dims) - {v["dimension"] for v in videos}
    if missing:
        raise ValueError(f"the metadata has no prompts for {sorted(missing)}")
    return _seal(dict(schema=PROTOCOL_SCHEMA, repository=VBENCH_REPOSITORY, revision=VBENCH_REVISION,
                      version=VBENCH_VERSION, full_info_sha256=_sha_file(src), dimensions=dims,
                      settings=settings or {}, videos=videos,
                      note="what to generate; not a score and not a record of served requests"))


def export_videos(videos: dict, protocol: dict, videos_dir, fps: int = 16) -> dict:
    """``videos``: {(prompt, seed): tensor [3, T, H, W]} -> mp4 files at the protocol's paths."""
    import torch
    if not _sealed(protocol):
        raise ValueError("the generation protocol was altered")
    ffmpeg = shutil.which("ffmpeg")
    if ffmpeg is None:
        raise LookupError("ffmpeg is required to write VBench videos")
    out = Path(videos_dir)
    out.mkdir(parents=True, exist_ok=True)
    written = {}
    want = protocol["settings"]
    for rec in protocol["videos"]:
        key = (rec["prompt"], rec["seed"])
        if key not in videos:
            raise LookupError(f"no generated video for {rec['path']}")
        v = videos[key]
        if v.dim() != 4 or v.shape[0] != 3:
            raise ValueError(f"video for {rec['path']} is not [3, T, H, W]")
        if want and (v.shape[1], v.shape[2], v.shape[3]) != (want.get("frames"), want.get("height"), want.get("width")):
            raise ValueError(f"{rec['path']}: shape {tuple(v.shape)} differs from the generation settings")
        if v.dtype != torch.uint8:
            v = ((v.float().clamp(-1, 1) + 1) * 127.5).round().to(torch.uint8)
        target = out / rec["path"]
        target.parent.mkdir(parents=True, exist_ok=True)
        frames = v.permute(1, 2, 3, 0).contiguous().cpu().numpy()
        t, h, w, _ = frames.shape
        cmd = [ffmpeg, "-y", "-loglevel", "error", "-f", "rawvideo", "-pix_fmt", "rgb24", "-s", f"{w}x{h}", "-r",
               str(fps), "-i", "-", "-pix_fmt", "yuv420p", "-c:v", "libx264", str(target)]
        subprocess.run(cmd, input=frames.tobytes(), check=True, timeout=600)
        written[rec["path"]] = _sha_file(target)
    return dict(videos=len(written), sha256=written)


def _checkout(repo: Path, timeout: float) -> tuple[str, bool]:
    git = shutil.which("git")
    if git is None:
        raise LookupError("git is required to verify the VBench checkout")
    head = subprocess.run([git, "-C", str(repo), "rev-parse", "HEAD"], capture_output=True, text=True,
                          timeout=timeout, check=True).stdout.strip()
    dirty = subprocess.run([git, "-C", str(repo), "status", "--porcelain", "--untracked-files=no"],
                           capture_output=True, text=True, timeout=timeout, check=True).stdout.strip()
    return head, bool(dirty)


def run_vbench(protocol_path, videos_dir, repo_dir, output_dir=None, python=None, timeout: float = 3600.0,
               video_hashes: dict | None = None) -> dict:
    deadline = time.monotonic() + timeout

    def left():
        r = deadline - time.monotonic()
        if r <= 0:
            raise TimeoutError("the VBench evaluation deadline ran out")
        return r
    protocol = json.loads(Path(protocol_path).read_text())
    if protocol.get("schema") != PROTOCOL_SCHEMA or protocol.get("revision") != VBENCH_REVISION:
        raise ValueError("not a generation protocol for the pinned VBench revision")
    if not _sealed(protocol):
        raise ValueError("the generation protocol was altered")
    repo = Path(repo_dir)
    if not (repo / "evaluate.py").is_file():
        raise LookupError(f"no VBench checkout at {repo}")
    head, dirty = _checkout(repo, left())
    if head != VBENCH_REVISION or dirty:
        raise ValueError(f"VBench checkout at {head[:12]} (dirty={dirty}) is not the pinned {VBENCH_REVISION[:12]}")
    videos = Path(videos_dir)
    for rec in protocol["videos"]:
        p = videos / rec["path"]
        if not p.is_file():
            raise LookupError(f"missing video {rec['path']}")
        if video_hashes is not None and video_hashes.get(rec["path"]) != _sha_file(p):
            raise ValueError(f"video {rec['path']} changed since export")
    out = Path(output_dir) if output_dir else videos / "vbench_results"
    out.mkdir(parents=True, exist_ok=True)
    scores = {}
    for dim in protocol["dimensions"]:
        expect = sum(1 for r in protocol["videos"] if r["dimension"] == dim)
        cmd = [python or sys.executable, str(repo / "evaluate.py"), "--videos_path", str(videos / dim),
               "--dimension", dim, "--output_path", str(out / dim)]
        proc = subprocess.run(cmd, cwd=str(repo), capture_output=True, text=True, timeout=left(),
                              env=dict(os.environ, PYTHONPATH=str(repo)))
        results = sorted((out / dim).glob("*_eval_results.json")) if (out / dim).exists() else []
        if proc.returncode != 0 or not results:
            raise RuntimeError(f"VBench {dim} failed: {proc.stderr[-2000:]}")
        res = json.loads(results[-1].read_text())
        entry = res.get(dim)
        if not isinstance(entry, list) or len(entry) < 2 or not isinstance(entry[1], list):
            raise ValueError(f"VBench {dim} wrote an unrecognised result")
        if len(entry[1]) != expect:
            raise ValueError(f"VBench {dim} scored {len(entry[1])} videos, the protocol has {expect}")
        scores[dim] = float(entry[0])
    return dict(revision=VBENCH_REVISION, protocol_seal=protocol["seal"], scores=scores)
