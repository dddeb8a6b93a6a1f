"""Fused peer-memory collectives on real GPUs.

* bounded waits: a barrier whose peer never signals returns a timeout status (1 GPU;
  the "peer" slot is a flag nothing sets) and the context stays usable;
* with >= 2 GPUs: the fused path equals the NCCL path bitwise (torchrun child processes).
"""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_barrier_times_out_and_reports_status():
    from ditserve_b200.ops import KernelTimeout, check_status, ext, status_word
    dev = torch.device("cuda", 0)
    heap, _ = ext().symm_alloc(1 << 20, 0)
    base = heap.data_ptr()
    st = status_word(dev)
    # a two-member group whose second member is this same heap: slot 1 is never written
    ext().group_barrier(0, [base, base], int(0.2e9), 3, 1, st)
    torch.cuda.synchronize()
    with pytest.raises(KernelTimeout, match="peer flag"):
        check_status(dev)
    # the context is still usable afterwards
    x = torch.ones(4, device=dev)
    assert float(x.sum()) == 4.0
    check_status(dev)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
def test_fused_equals_nccl_bitwise():
    n = 4 if torch.cuda.device_count() >= 4 else 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", "29533", "-m",
                        "ditserve_b200.parallel.selftest", "--tiny"], cwd=ROOT, capture_output=True, text=True,
                       env=env, timeout=460)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("{")][-1]
    res = json.loads(line)
    assert res["bitwise_equal_all_ranks"], json.dumps(res)


def test_group_flag_single_and_timeout():
    from ditserve_b200.ops import KernelTimeout, check_status, ext, status_word
    dev = torch.device("cuda", 0)
    heap, _ = ext().symm_alloc(1 << 20, 0)
    base = heap.data_ptr()
    st = status_word(dev)
    out = torch.zeros(1, dtype=torch.int32, device=dev)
    for f in (0, 1):  # a one-member group: the MAX is this rank's own flag, no wait
        ext().group_flag(0, [base], int(0.2e9), 5, 1 + f, f, out, st)
        assert int(out.item()) == f
    check_status(dev)
    # a second member that never signals: the wait expires, out = -1 and a status is recorded
    ext().group_flag(0, [base, base], int(0.2e9), 6, 1, 1, out, st)
    torch.cuda.synchronize()
    assert int(out.item()) == -1
    with pytest.raises(KernelTimeout, match="peer flag"):
        check_status(dev)
    assert float(torch.ones(3, device=dev).sum()) == 3.0


def test_put_peers_copies_bytes():
    from ditserve_b200.ops import ext
    heap, _ = ext().symm_alloc(8 << 20, 0)
    src = torch.randn(1 << 18, device="cuda")
    off = 1 << 20
    ext().put_peers(src, 1, off, 0, [heap.data_ptr()], int(1e9))
    torch.cuda.synchronize()
    got = heap[off:off + src.numel() * 4].view(torch.float32)
    assert torch.equal(got, src)
    with pytest.raises(RuntimeError):
        ext().put_peers(src[1:], 1, off, 0, [heap.data_ptr()], int(1e9))  # misaligned source


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
def test_elastic_paths_multi_gpu():
    n = 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", "29534", "-m",
                        "ditserve_b200.parallel.elastic_check", "--mb", "8"], cwd=ROOT, capture_output=True,
                       text=True, env=env, timeout=360)
    assert r.returncode == 0, r.stderr[-3000:]
    res = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    assert res["flags_agree"] and res["broadcast_bitwise"] and res["broadcast_ce_bitwise"], res

