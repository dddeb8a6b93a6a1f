"""Python client of the native controller (``ditserve-b200``).

    Client().rpc("plan", {...}) / Client().run(config, run_id=...) / Client().policies()

Requests go to ``ditserve-b200 rpc <command>`` on stdin; replies are parsed JSON.
Reference: workers/ditserve/runtime/client.py:15-96.
"""
from __future__ import annotations

import json
import os
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
DEFAULT_BINARY = ROOT / "cpp" / "controller" / "build" / "ditserve-b200"


class ControllerError(RuntimeError):
    pass


class Client:
    def __init__(self, binary: str | os.PathLike | None = None, timeout: float = 3600):
        self.binary = str(binary or os.environ.get("DITSERVE_CORE", DEFAULT_BINARY))
        self.timeout = timeout

    def rpc(self, command: str, request: dict) -> dict:
        env = dict(os.environ)
        env.setdefault("DITSERVE_PACKAGE_ROOT", str(ROOT))
        r = subprocess.run([self.binary, "rpc", command], input=json.dumps(request), capture_output=True, text=True,
                           timeout=self.timeout, env=env)
        if r.returncode != 0:
            raise ControllerError(f"rpc {command} failed ({r.returncode}): {r.stderr.strip()}")
        return json.loads(r.stdout)

    def policies(self):
        return self.rpc("policies", {})

    def plan(self, state: dict, policy: str = "ditserve", options: dict | None = None, profile: dict | None = None):
        req = dict(state=state, policy=policy, options=options or {})
        if profile is not None:
            req["profile"] = profile
        return self.rpc("plan", req)

    def simulate(self, phase: dict):
        return self.rpc("simulate", phase)

    def run(self, config: dict, run_id: str, work_dir: str = "runs", allow_gpu: bool = False, resume: bool = False):
        return self.rpc("run", dict(config=config, run_id=run_id, work_dir=work_dir, allow_gpu=allow_gpu,
                                    resume=resume))
