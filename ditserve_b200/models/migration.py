"""Cross-device request migration and read-only state inventory.

Two-phase protocol between a source and a target backend (each a worker in practice):

    1. source.pause   -> exports a packet (bytes + SHA-256 manifest) at a step/block boundary;
                         the source keeps the state, marked paused, under a migration epoch
    2. target.prepare -> imports and verifies the packet, holds it uncommitted
    3. ack            -> the coordinator checks both sides agree on (state_id, epoch, digest)
    4. source.release -> the source drops its copy
    5. target.commit  -> the target makes the state live
Abort before step 4 restores the source (unpause) and drops the target's copy; after a
failed commit the source copy is gone, so the target keeps its verified packet and can
retry the commit.  Epochs reject stale or replayed messages.  ``local_roundtrip`` runs
the protocol between two engines in one process (the control experiment).

``inventory`` / ``refresh_certificate`` describe a state without touching its values:
tensor descriptors (shape, dtype, device, byte size) and a version-bound certificate
(model + scheduler kinds + progress) that a resumed request must present.
Reference: workers/ditserve/models/wan/migration.py:179-514, state.py:105-368.
"""
from __future__ import annotations

import hashlib
import json

import torch


class MigrationError(RuntimeError):
    pass


class MigrationEndpoint:
    """Wraps an engine (WanEngine-like: export_packet/import_packet) and its live states."""

    def __init__(self, engine, states: dict):
        self.engine = engine
        self.states = states
        self.paused: dict = {}    # state_id -> (epoch, digest)
        self.pending: dict = {}   # state_id -> (epoch, digest, state)

    # source side
    def pause(self, state_id: str, epoch: int):
        st = self.states.get(state_id)
        if st is None:
            raise MigrationError(f"unknown state {state_id}")
        if state_id in self.paused:
            raise MigrationError("state is already being migrated")
        blob, digest = self.engine.export_packet(st)
        self.paused[state_id] = (epoch, digest)
        return dict(state_id=state_id, epoch=epoch, digest=digest, packet=blob)

    def release(self, state_id: str, epoch: int, digest: str):
        e = self.paused.get(state_id)
        if e is None or e != (epoch, digest):
            raise MigrationError("release does not match the paused migration")
        del self.paused[state_id]
        del self.states[state_id]

    def abort(self, state_id: str, epoch: int):
        e = self.paused.get(state_id)
        if e is not None and e[0] == epoch:
            del self.paused[state_id]
        p = self.pending.get(state_id)
        if p is not None and p[0] == epoch:
            del self.pending[state_id]

    # target side
    def prepare(self, state_id: str, epoch: int, digest: str, packet: bytes):
        if state_id in self.states or state_id in self.pending:
            raise MigrationError("target already holds this state")
        st = self.engine.import_packet(packet, digest)
        self.pending[state_id] = (epoch, digest, st)
        return dict(state_id=state_id, epoch=epoch, digest=digest)

    def commit(self, state_id: str, epoch: int, digest: str):
        p = self.pending.get(state_id)
        if p is None or p[:2] != (epoch, digest):
            raise MigrationError("commit does not match the prepared migration")
        self.states[state_id] = p[2]
        del self.pending[state_id]
        return dict(state_id=state_id, epoch=epoch, committed=True)


def migrate(source: MigrationEndpoint, target: MigrationEndpoint, state_id: str, epoch: int,
            fail_after: str | None = None) -> dict:
    """Run the protocol; ``fail_after`` (pause|prepare|ack) injects a host-side failure."""
    pkt = source.pause(state_id, epoch)
    try:
        if fail_after == "pause":
            raise MigrationError("injected failure after pause")
        ack = target.prepare(state_id, epoch, pkt["digest"], pkt["packet"])
        if fail_after == "prepare":
            raise MigrationError("injected failure after prepare")
        if (ack["state_id"], ack["epoch"], ack["digest"]) != (state_id, epoch, pkt["digest"]):
            raise MigrationError("target acknowledged a different migration")
        if fail_after == "ack":
            raise MigrationError("injected failure after ack")
    except Exception:
        source.abort(state_id, epoch)
        target.abort(state_id, epoch)
        raise
    source.release(state_id, epoch, pkt["digest"])
    return target.commit(state_id, epoch, pkt["digest"])


def local_roundtrip(engine, state, epoch: int = 1) -> object:
    """Migrate a state out of and back into the same engine (protocol overhead control)."""
    a = MigrationEndpoint(engine, {"x": state})
    b = MigrationEndpoint(engine, {})
    migrate(a, b, "x", epoch)
    return b.states["x"]


def _describe(t) -> dict:
    if isinstance(t, torch.Tensor):
        return dict(shape=list(t.shape), dtype=str(t.dtype).replace("torch.", ""), device=str(t.device),
                    bytes=t.numel() * t.element_size())
    return None


def inventory(state) -> dict:
    """Read-only schema of a Wan/SD3.5 request state: descriptors, never values."""
    out = dict(kind=type(state).__name__, step=getattr(state, "step", None))
    spec = getattr(state, "spec", None)
    if spec is not None and hasattr(spec, "to_dict"):
        out["spec"] = spec.to_dict()
    tensors = {}
    for name in ("latents", "context", "negative", "pooled", "neg_context", "neg_pooled"):
        d = _describe(getattr(state, name, None))
        if d is not None:
            tensors[name] = d
    sched = getattr(state, "scheduler", None)
    if sched is not None:
        sd = sched.state_dict(device=None) if "device" in sched.state_dict.__code__.co_varnames else sched.state_dict()
        out["scheduler"] = {k: v for k, v in sd.items() if not isinstance(v, (torch.Tensor, list)) or k == "hist_sigmas"}
        for i, t in enumerate(sd.get("hist", []) or []):
            tensors[f"scheduler.hist.{i}"] = _describe(t)
        if sd.get("last") is not None:
            tensors["scheduler.last"] = _describe(sd["last"])
    out["tensors"] = tensors
    out["bytes"] = sum(d["bytes"] for d in tensors.values())
    return out


def refresh_certificate(state, model_version: str) -> dict:
    """Version-bound certificate of a state's identity; a resume must present a matching one."""
    inv = inventory(state)
    body = dict(model_version=model_version, kind=inv["kind"], step=inv["step"], spec=inv.get("spec"),
                scheduler=inv.get("scheduler", {}).get("kind"),
                tensors={k: [v["shape"], v["dtype"]] for k, v in inv["tensors"].items()})
    digest = hashlib.sha256(json.dumps(body, sort_keys=True).encode()).hexdigest()
    return dict(body, certificate=digest)


def check_certificate(state, model_version: str, cert: dict) -> bool:
    return refresh_certificate(state, model_version)["certificate"] == cert.get("certificate")
