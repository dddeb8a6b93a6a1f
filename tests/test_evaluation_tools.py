"""VBench protocol and pinned-checkout refusals, offline dataset prep, all-to-all microbench (CPU)."""
import csv
import json
import os
import shutil
import socket
import subprocess

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ditserve_b200.evaluation import datasets, vbench


def _full_info(tmp_path):
    info = [{"prompt_en": "a cat surfing", "dimension": ["subject_consistency", "temporal_flickering"]},
            {"prompt_en": "a red car", "dimension": ["color", "subject_consistency"]}]
    p = tmp_path / "VBench_full_info.json"
    p.write_text(json.dumps(info))
    return p


def test_vbench_generation_protocol(tmp_path):
    proto = vbench.generation_protocol(_full_info(tmp_path), ["subject_consistency", "temporal_flickering"],
                                       settings={"frames": 81, "height": 480, "width": 832})
    per = {}
    for v in proto["videos"]:
        per[v["dimension"]] = per.get(v["dimension"], 0) + 1
    assert per == {"subject_consistency": 10, "temporal_flickering": 25}
    assert proto["videos"][0]["path"] == "subject_consistency/a cat surfing-0.mp4"
    assert vbench._sealed(proto)
    with pytest.raises(ValueError):
        vbench.generation_protocol(_full_info(tmp_path), ["color", "scene"])   # no prompts for "scene"
    with pytest.raises(ValueError):
        vbench.generation_protocol(_full_info(tmp_path), ["not_a_dimension"])


@pytest.mark.skipif(shutil.which("git") is None, reason="git not installed")
def test_vbench_refuses_missing_or_unpinned_checkouts(tmp_path):
    proto = vbench.generation_protocol(_full_info(tmp_path), ["color"])
    pp = tmp_path / "protocol.json"
    pp.write_text(json.dumps(proto))
    with pytest.raises(LookupError):
        vbench.run_vbench(pp, tmp_path / "videos", tmp_path / "no_checkout")
    repo = tmp_path / "VBench"
    repo.mkdir()
    (repo / "evaluate.py").write_text("print('not the official evaluator')\n")
    env = dict(os.environ, GIT_AUTHOR_NAME="t", GIT_AUTHOR_EMAIL="t@t", GIT_COMMITTER_NAME="t",
               GIT_COMMITTER_EMAIL="t@t")
    subprocess.run(["git", "init", "-q", str(repo)], check=True, env=env)
    subprocess.run(["git", "-C", str(repo), "add", "."], check=True, env=env)
    subprocess.run(["git", "-C", str(repo), "commit", "-qm", "x"], check=True, env=env)
    with pytest.raises(ValueError, match="not the pinned"):
        vbench.run_vbench(pp, tmp_path / "videos", repo)
    tampered = dict(proto, dimensions=["color", "scene"])
    pp.write_text(json.dumps(tampered))
    with pytest.raises(ValueError, match="altered"):
        vbench.run_vbench(pp, tmp_path / "videos", repo)


def test_dataset_prep_vbench_and_vidprom(tmp_path):
    m = datasets.prepare_dataset("vbench", _full_info(tmp_path), dev_count=1)
    assert [s["split"] for s in m["samples"]] == ["evaluation", "evaluation"]
    assert sorted(s["role"] for s in m["samples"]) == ["dev", "test"]
    csv_path = tmp_path / "vidprom.csv"
    with csv_path.open("w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=["uuid", "prompt", "time", "toxicity", "sexual_explicit"])
        w.writeheader()
        for i in range(200):
            w.writerow({"uuid": f"u{i}", "prompt": f"scene number {i % 150}", "time": f"2024-01-{i % 28 + 1:02d}",
                        "toxicity": 0.9 if i % 10 == 0 else 0.1, "sexual_explicit": ""})
    a = datasets.prepare_dataset("vidprom", csv_path, dev_count=5, sample_count=40, seed=7)
    b = datasets.prepare_dataset("vidprom", csv_path, dev_count=5, sample_count=40, seed=7)
    assert a == b and len(a["samples"]) == 40 and a["rows_skipped"] == 20
    assert all("u0" != s["sample_id"][len("vidprom-"):] for s in a["samples"])  # unsafe row 0 dropped
    # duplicates of one prompt never straddle the roles
    by_text = {}
    for s in a["samples"]:
        by_text.setdefault(s["prompt"].lower(), set()).add(s["role"])
    assert all(len(r) == 1 for r in by_text.values())
    c = datasets.prepare_dataset("vidprom", csv_path, dev_count=5, sample_count=40, seed=8)
    assert c["samples"] != a["samples"]
    with pytest.raises(ValueError):
        datasets.prepare_dataset("vidprom", csv_path, expected_sha256="0" * 64)
    with pytest.raises(LookupError):
        datasets.prepare_dataset("diffusiondb", tmp_path / "missing.parquet")


def test_dataset_prep_diffusiondb_parquet(tmp_path):
    import pyarrow as pa
    import pyarrow.parquet as pq
    rows = [{"image_name": f"{i}.png", "prompt": f"photo {i}", "prompt_nsfw": 0.7 if i < 3 else 0.01}
            for i in range(30)]
    pq.write_table(pa.Table.from_pylist(rows), tmp_path / "metadata.parquet")
    m = datasets.prepare_dataset("diffusiondb", tmp_path / "metadata.parquet", dev_count=4, sample_count=10)
    assert len(m["samples"]) == 10 and m["rows_skipped"] == 3 and m["roles"] == {"dev": 4, "test": 6}


def _a2a_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ditserve_b200.evaluation.collectives import measure
        rows = measure(sizes_mb=(0.25, 1), iterations=2, warmup=1, device=torch.device("cpu"))
        if rank == 0:
            out["rows"] = rows
    finally:
        dist.destroy_process_group()


def test_all_to_all_microbench_gloo():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = mp.Manager().dict()
    mp.spawn(_a2a_worker, args=(2, port, out), nprocs=2, join=True)
    rows = out["rows"]
    assert [r["size_mb"] for r in rows] == [0.25, 1] and all(r["algbw_gbs"] > 0 for r in rows)
    assert rows[1]["busbw_gbs"] == pytest.approx(rows[1]["algbw_gbs"] / 2, rel=0.02)
