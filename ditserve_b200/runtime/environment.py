"""`doctor` metadata without initialising CUDA (safe on a busy or absent GPU)."""
from __future__ import annotations

import os
import platform
import shutil
import subprocess
import sys


def environment() -> dict:
    out = dict(python=sys.version.split()[0], platform=platform.platform(), cpus=os.cpu_count())
    try:
        import torch
        out["torch"] = torch.__version__
        out["torch_cuda"] = torch.version.cuda
        out["nccl"] = ".".join(map(str, torch.cuda.nccl.version())) if hasattr(torch.cuda, "nccl") else None
    except Exception as exc:  # noqa: BLE001
        out["torch"] = f"unavailable: {exc}"
    from ..ops import _ext
    out["extension_built"] = _ext.available()
    nvcc = shutil.which("nvcc")
    if nvcc:
        r = subprocess.run([nvcc, "--version"], capture_output=True, text=True)
        out["nvcc"] = r.stdout.strip().splitlines()[-1] if r.returncode == 0 else None
    smi = shutil.which("nvidia-smi")
    if smi:
        r = subprocess.run([smi, "--query-gpu=index,name,memory.total,clocks.max.sm", "--format=csv,noheader"],
                           capture_output=True, text=True, timeout=10)
        out["gpus"] = r.stdout.strip().splitlines() if r.returncode == 0 else []
    else:
        out["gpus"] = []
    return out


class EnvironmentBackend:
    operations = ("doctor",)

    def __init__(self, config):
        self.config = config
        self.states = {}

    def capabilities(self):
        return {}

    def doctor(self, request):
        return environment()

    def close(self):
        pass
