"""Protocol v1 framing: one strict JSON object per line.

request : {"version": 1, "id": <int|str>, "op": <str>, ...fields}
reply   : {"version": 1, "id": <same>, "ok": true, "result": {...}}
        | {"version": 1, "id": <same>, "ok": false, "error": "<message>", "error_type": "<class>"}
NaN/Infinity are rejected in both directions (they are not JSON).
Reference envelope: workers/ditserve/runtime/worker.py:108-118, :393-423.
"""
from __future__ import annotations

import json

from . import PROTOCOL_VERSION


class ProtocolError(ValueError):
    pass


def _reject_constant(name):
    raise ProtocolError(f"non-finite JSON constant {name}")


def loads(line: str):
    try:
        return json.loads(line, parse_constant=_reject_constant)
    except json.JSONDecodeError as exc:
        raise ProtocolError(f"invalid JSON: {exc}") from None


def dumps(obj) -> str:
    return json.dumps(obj, allow_nan=False, separators=(",", ":"), sort_keys=True)


def operation(request) -> str:
    if not isinstance(request, dict):
        raise ProtocolError("request must be a JSON object")
    if request.get("version") != PROTOCOL_VERSION:
        raise ProtocolError(f"unsupported protocol version {request.get('version')!r}")
    if "id" not in request or not isinstance(request["id"], (int, str)) or isinstance(request["id"], bool):
        raise ProtocolError("request needs an integer or string id")
    op = request.get("op")
    if not isinstance(op, str) or not op:
        raise ProtocolError("request needs an op")
    return op


def ok(request_id, result) -> dict:
    return {"version": PROTOCOL_VERSION, "id": request_id, "ok": True, "result": result}


def error(request_id, exc: BaseException) -> dict:
    return {"version": PROTOCOL_VERSION, "id": request_id, "ok": False, "error": str(exc) or type(exc).__name__,
            "error_type": type(exc).__name__}
