"""Deterministic CPU fixture backend (no model, no GPU).

The "latent" is a SHA-256 chain: each solver step hashes the previous value,
so any schedule of step/block quanta, snapshots, exports and migrations that
is exact ends on the same digest as an uninterrupted run.  It implements every
op of the real backends so the controller, the study runner and the failure
paths can be tested on CPU:

* step and block quanta (blocks_per_step > 1), doorbell stops at check_blocks
  boundaries, lockstep pairs (pair_state_id), continuous image batches
  (advance_batch with late joins and early exits);
* snapshot / restore (hot or cold), block_export / block_import packets with a
  SHA-256 manifest (tampering is rejected), two-phase migration release/abort;
* encode / decode tickets with optional delays;
* host-side fault injection: options or request ``inject`` = {fail_on: op,
  fail_ops: [ops], delay_ms, print: text (stdout pollution)}; costs.step_ms /
  prepare_ms make it sleep like a model would.

Reference fixture: workers/ditserve/models/mock.py:11-486.
"""
from __future__ import annotations

import hashlib
import json
import time

from ..runtime.doorbell import rung
from .base import Backend, artifact, positive_int, progress


def _chain(value: str) -> str:
    return hashlib.sha256(value.encode()).hexdigest()


class MockBackend(Backend):
    operations = Backend.operations + (
        "snapshot", "restore", "inventory", "distributed", "advance_batch", "generate_batch",
        "encode_start", "encode_poll", "encode_discard", "decode_start", "decode_poll",
        "block_export", "block_import", "migration_release", "migration_abort")

    def __init__(self, config):
        super().__init__(config)
        self.tickets: dict = {}
        self.decodes: dict = {}
        self.exports: dict = {}
        self.mid_step = None
        self.world = None

    def capabilities(self):
        return dict(quanta=["step", "blocks"], migration=True, sp_degrees=[1, 2, 3, 4, 6, 8],
                    continuous_batch=8, fixture=True)

    # -------------------------------------------------------------- helpers
    def _inject(self, op, request):
        opts = dict(self.config.get("options", {}))
        opts.update(request.get("inject", {}) or {})
        delay = opts.get("delay_ms", 0)
        if type(delay) not in (int, float) or not 0 <= delay <= 60000:
            raise ValueError("delay_ms must be in [0, 60000]")
        if delay:
            time.sleep(delay / 1000)
        if opts.get("print"):
            print(opts["print"])  # goes to stderr: the worker re-routes stdout
        if op == opts.get("fail_on") or op in opts.get("fail_ops", []):
            raise RuntimeError(f"injected mock {op} failure")

    def _sleep(self, key, scale=1.0):
        ms = self.config.get("options", {}).get("costs", {}).get(key, 0) * scale
        if type(ms) not in (int, float) or not 0 <= ms <= 60000:
            raise ValueError("mock costs must be in [0, 60000] ms")
        if ms:
            time.sleep(ms / 1000)

    @staticmethod
    def _progress(st):
        p = progress(st["step"], st["steps"])
        if st["blocks"] > 1:
            p.update(block=st["unit"] % st["blocks"], transfer_ready=st["unit"] % st["blocks"] == 0)
        return p

    # -------------------------------------------------------------- lifecycle
    def prepare(self, request):
        self._inject("prepare", request)
        key = self.new_id(request)
        spec = dict(request.get("spec", {}))
        if request.get("encode_ticket"):
            t = request["encode_ticket"]
            if t not in self.tickets:
                raise ValueError("unknown encode ticket")
            enc_spec, ready_at = self.tickets.pop(t)
            if time.monotonic() < ready_at:
                raise ValueError("encode ticket is not ready")
        steps = positive_int(spec.get("steps", 2))
        blocks = positive_int(spec.get("blocks_per_step", 1), "blocks_per_step")
        seed = spec.get("seed", 0)
        if type(seed) is not int or seed < 0:
            raise ValueError("seed must be a nonnegative integer")
        value = hashlib.sha256(json.dumps({"prompt": spec.get("prompt", ""), "seed": seed},
                                          sort_keys=True).encode()).hexdigest()
        resume = request.get("resume", {}) or {}
        unit = int(resume.get("step", 0)) * blocks + int(resume.get("block", 0))
        if not 0 <= unit < steps * blocks:
            raise ValueError("resume position is outside the request")
        # resuming re-derives the chain position (exactly what a restored state would hold)
        for _ in range(unit // blocks):
            value = _chain(value)
        self.states[key] = dict(step=unit // blocks, steps=steps, unit=unit, blocks=blocks, value=value,
                                paused=False, residency="device", kind=spec.get("kind", "video"))
        self._sleep("prepare_ms")
        return dict(state_id=key, progress=self._progress(self.states[key]), measured=False)

    def advance(self, request):
        pair = request.get("pair_state_id")
        if pair is not None:
            if pair == request.get("state_id") or pair not in self.states:
                raise ValueError("unknown pair_state_id")
            a = self._advance_one(dict(request, pair_state_id=None), partner=pair)
            b = self._advance_one(dict(request, state_id=pair, pair_state_id=None), partner=request["state_id"])
            return dict(a, pair_state_id=pair, pair_progress=b["progress"])
        return self._advance_one(request)

    def _advance_one(self, request, partner=None):
        self._inject("advance", request)
        st = self.state(request)
        if st["paused"]:
            raise ValueError("restore the state before advancing")
        if st["step"] >= st["steps"]:
            raise ValueError("request has no remaining steps")
        degree = positive_int(request.get("sp_degree", 1), "sp_degree")
        grouped = "epoch" in request and st["blocks"] > 1
        if grouped and self.mid_step not in (None, request["state_id"], partner):
            raise ValueError("another request is inside a solver step on this worker")
        placement = [list(request.get("group") or []), request.get("epoch")]
        if grouped and st["unit"] % st["blocks"] and st.get("placement") not in (None, placement):
            raise ValueError("the SP group may change only at a solver-step boundary")
        t0 = time.perf_counter()
        stopped = False
        if st["blocks"] == 1:
            n = positive_int(request.get("steps", request.get("blocks", 1)))
            done = min(n, st["steps"] - st["step"])
            for _ in range(done):
                st["value"] = _chain(st["value"])
                st["step"] += 1
            st["unit"] = st["step"]
            self._sleep("step_ms", done / degree)
        else:
            boundary = st["blocks"] - st["unit"] % st["blocks"]
            want = boundary if request.get("quantum") == "step" else min(positive_int(request.get("blocks", 1)), boundary)
            bell = rung(request)
            check = positive_int(request.get("check_blocks", 1), "check_blocks")
            done = 0
            while done < want:
                chunk = min(check, want - done)
                self._sleep("step_ms", chunk / st["blocks"] / degree)
                done += chunk
                if done < want and bell is not None and bell():
                    stopped = True
                    break
            st["unit"] += done
            if st["unit"] % st["blocks"] == 0:
                st["value"] = _chain(st["value"])
            st["step"] = st["unit"] // st["blocks"]
            if grouped:
                st["placement"] = placement if st["unit"] % st["blocks"] else None
                self.mid_step = request["state_id"] if st["unit"] % st["blocks"] else None
        return dict(state_id=request["state_id"], executed=done, doorbell_stop=stopped,
                    progress=self._progress(st), model_ms=(time.perf_counter() - t0) * 1000, measured=False)

    def advance_batch(self, request):
        """One denoise step for every member (continuous batching); members may join or leave."""
        self._inject("advance_batch", request)
        out = []
        for sid in request["state_ids"]:
            st = self.state(dict(state_id=sid))
            if st["step"] < st["steps"]:
                st["value"] = _chain(st["value"])
                st["step"] += 1
                st["unit"] = st["step"] * st["blocks"]
            out.append(dict(state_id=sid, progress=self._progress(st)))
        self._sleep("step_ms", 1.0)
        return dict(members=out, batch=len(out), measured=False)

    def generate_batch(self, request):
        res = []
        for spec in request["specs"]:
            sid = self.prepare(dict(request, spec=spec, state_id=spec["request_id"]))["state_id"]
            st = self.states[sid]
            while st["step"] < st["steps"]:
                self._advance_one(dict(id=request["id"], state_id=sid, steps=st["steps"]))
            res.append(self.finish(dict(request, state_id=sid)))
            self.release(dict(state_id=sid))
        return dict(results=res)

    def finish(self, request):
        self._inject("finish", request)
        st = self.state(request)
        if st["step"] != st["steps"]:
            raise ValueError("request is not complete")
        mode = request.get("output_mode", "digest")
        data = [int(st["value"][i:i + 2], 16) for i in range(0, 64, 2)]
        art = artifact(data, self.output_path(request) if mode == "file" else None, mode)
        return dict(state_id=request["state_id"], value=st["value"], artifact=art, measured=False)

    def inventory(self, request):
        return dict(states={k: dict(step=v["step"], steps=v["steps"], unit=v["unit"], paused=v["paused"],
                                    residency=v["residency"]) for k, v in self.states.items()})

    # -------------------------------------------------------------- state movement
    def snapshot(self, request):
        self._inject("snapshot", request)
        st = self.state(request)
        mode = request.get("mode", "hot")
        if mode not in ("hot", "cold", "keep"):
            raise ValueError("snapshot mode must be hot, cold or keep")
        if mode != "keep":
            st["paused"] = True
            st["residency"] = "host" if mode == "hot" else "disk"
        return dict(state_id=request["state_id"], mode=mode, progress=self._progress(st), value=st["value"])

    def restore(self, request):
        st = self.state(request)
        st["paused"] = False
        st["residency"] = "device"
        return dict(state_id=request["state_id"], progress=self._progress(st))

    def block_export(self, request):
        self._inject("block_export", request)
        st = self.state(request)
        packet = dict(state=dict(st, placement=None), state_id=request["state_id"])
        body = json.dumps(packet, sort_keys=True)
        manifest = hashlib.sha256(body.encode()).hexdigest()
        self.exports[request["state_id"]] = manifest
        return dict(packet=body, manifest=manifest, bytes=len(body))

    def block_import(self, request):
        self._inject("block_import", request)
        body = request["packet"]
        if hashlib.sha256(body.encode()).hexdigest() != request["manifest"]:
            raise ValueError("packet manifest mismatch (tampered or truncated transfer)")
        packet = json.loads(body)
        key = request.get("state_id", packet["state_id"])
        if key in self.states:
            raise ValueError("duplicate live state_id")
        self.states[key] = dict(packet["state"])
        return dict(state_id=key, progress=self._progress(self.states[key]))

    def migration_release(self, request):
        self.state(request)
        del self.states[request["state_id"]]
        self.exports.pop(request["state_id"], None)
        return dict(released=request["state_id"])

    def migration_abort(self, request):
        st = self.state(request)
        st["paused"] = False
        self.exports.pop(request["state_id"], None)
        return dict(aborted=request["state_id"])

    # -------------------------------------------------------------- tickets
    def encode_start(self, request):
        ticket = f"encode-{request['id']}"
        delay = self.config.get("options", {}).get("encode_delay_ms", 0)
        self.tickets[ticket] = (dict(request.get("spec", {})), time.monotonic() + delay / 1000)
        return dict(ticket=ticket, ready=False, measured=False)

    def encode_poll(self, request):
        if request["ticket"] not in self.tickets:
            raise ValueError("unknown encode ticket")
        return dict(ticket=request["ticket"], ready=time.monotonic() >= self.tickets[request["ticket"]][1])

    def encode_discard(self, request):
        self.tickets.pop(request.get("ticket"), None)
        return dict(discarded=True)

    def decode_start(self, request):
        st = self.state(request)
        if st["step"] != st["steps"]:
            raise ValueError("decode requires a completed state")
        delay = self.config.get("options", {}).get("decode_delay_ms", 0)
        ticket = f"decode-{request['id']}"
        self.decodes[ticket] = (request["state_id"], time.monotonic() + delay / 1000, dict(request))
        return dict(ticket=ticket, ready=False, state_id=request["state_id"])

    def decode_poll(self, request):
        if request["ticket"] not in self.decodes:
            raise ValueError("unknown decode ticket")
        sid, ready_at, orig = self.decodes[request["ticket"]]
        left = ready_at - time.monotonic()
        if left > 0 and not request.get("wait"):
            return dict(ticket=request["ticket"], ready=False, state_id=sid)
        if left > 0:
            time.sleep(left)
        res = self.finish(dict(orig, **{k: v for k, v in request.items() if k != "ticket"}, state_id=sid))
        del self.decodes[request["ticket"]]
        return dict(res, ticket=request["ticket"], ready=True)

    def distributed(self, request):
        action = request.get("action", "init")
        if action == "init":
            self.world = dict(rank=request.get("rank", 0), world_size=request.get("world_size", 1))
            return dict(initialised=True, **self.world)
        if action == "layout":  # the fixture has no collectives: record the layout only
            self.layout = dict(form=request["form"], ranks=list(request["ranks"]))
            return dict(self.layout, epoch=int(request.get("epoch", 0)))
        if action == "shutdown":
            self.world = None
            return dict(shutdown=True)
        raise ValueError(f"unknown distributed action {action!r}")
