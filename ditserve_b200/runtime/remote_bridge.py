"""Multi-node bridge: a worker on another node behind a local stand-in process.

    # node 1 (the GPUs): serve workers over TCP
    python -m ditserve_b200.runtime.remote_bridge daemon --listen 0.0.0.0:7700 --token "$SECRET"
    # node 0 (controller): a process that speaks the worker protocol on stdin/stdout
    python -m ditserve_b200.runtime.remote_bridge proxy --connect node1:7700 --backend wan --config '{...}'

Framing on the wire: 4-byte big-endian length + one JSON document, TCP_NODELAY.
The first frame of a connection is {"bridge": "spawn", "backend", "config", "env"}; the
daemon starts a local worker in a private session directory (always the worker's
``transfer_dir``; ``env`` may set CUDA_VISIBLE_DEVICES and
NCCL_* / DITSERVE_* variables) and relays protocol lines both ways.  Extra frames:
* {"bridge": "ring", "slot", "epoch"} — doorbell mirroring: the proxy watches the
  controller's local doorbell files and the daemon writes the epoch into its own
  copy, so a remote block quantum stops at its next check like a local one;
* {"bridge": "put_file", "name", "offset", "data_b64", "last"} /
  {"bridge": "get_file", "path", "offset", "unlink"} — chunked file staging, confined to
  the session directory;
* {"bridge": "occupancy", "gpus", "own_pids"} — the remote node's GPU occupancy probe (the
  session's worker counts as ours); the proxy answers the protocol op ``bridge_occupancy``
  with it, which is how the cluster executor's occupancy guard covers remote slots.
Requests naming a doorbell get the path rewritten to the daemon-side mirror.  Continuation
packets cross the bridge transparently: a ``block_export`` reply's packet file is fetched
into the proxy's staging directory (and removed remotely) and a ``block_import`` of a
local packet file is first pushed into the session directory, so the controller moves
state between a local and a remote worker, or between two nodes, exactly as between two
local workers.

The daemon runs whatever worker a client asks for: bind it to a cluster-internal address and
give it a shared secret (``--token`` or ``DITSERVE_BRIDGE_TOKEN``); a connection whose spawn
frame carries another token is closed before anything starts.  Without a token the daemon
refuses to listen on anything but a loopback address.  The remote worker's ``transfer_dir``
is always its session directory (a value in the client's config is replaced), so the file
frames never reach beyond the session.
Reference: workers/ditserve/runtime/remote_bridge.py:1-1009.
"""
from __future__ import annotations

import argparse
import base64
import hmac
import json
import os
import shutil
import socket
import struct
import subprocess
import sys
import tempfile
import threading
import time

from .doorbell import Doorbell


CHUNK = 8 << 20   # raw bytes per file-staging frame (base64 keeps a frame well under the 64 MiB cap)


def _is_loopback(host: str) -> bool:
    """True when every address ``host`` resolves to is a loopback address."""
    import ipaddress
    try:
        infos = socket.getaddrinfo(host, None)
    except OSError:
        return False
    addrs = {info[4][0] for info in infos}
    return bool(addrs) and all(ipaddress.ip_address(a.split("%")[0]).is_loopback for a in addrs)


def send_frame(sock: socket.socket, obj) -> None:
    data = json.dumps(obj, allow_nan=False).encode()
    sock.sendall(struct.pack(">I", len(data)) + data)


def recv_frame(sock: socket.socket):
    head = _recv_exact(sock, 4)
    if head is None:
        return None
    (n,) = struct.unpack(">I", head)
    if n > (64 << 20):
        raise ValueError("bridge frame exceeds 64 MiB")
    body = _recv_exact(sock, n)
    return None if body is None else json.loads(body)


def _recv_exact(sock, n):
    buf = bytearray()
    while len(buf) < n:
        chunk = sock.recv(n - len(buf))
        if not chunk:
            return None
        buf.extend(chunk)
    return bytes(buf)


class BridgeDaemon:
    """Accepts connections; each one gets its own local worker subprocess."""

    def __init__(self, host: str = "127.0.0.1", port: int = 0, python: str = sys.executable, workdir: str | None = None,
                 token: str | None = None):
        token = token if token is not None else os.environ.get("DITSERVE_BRIDGE_TOKEN")
        if not token and not _is_loopback(host):
            # the daemon starts whatever worker a client asks for: off the loopback interface
            # only a client holding the shared secret may do that
            raise ValueError(f"refusing to listen on {host!r} without a token: set --token or "
                             "DITSERVE_BRIDGE_TOKEN, or bind to a loopback address")
        self.server = socket.create_server((host, port))
        self.port = self.server.getsockname()[1]
        self.python = python
        self.workdir = workdir or tempfile.mkdtemp(prefix="ds-bridge-")
        os.makedirs(self.workdir, exist_ok=True)
        self.threads = []
        self._stop = threading.Event()
        self.token = token

    def serve_forever(self):
        self.server.settimeout(0.2)
        while not self._stop.is_set():
            try:
                conn, _ = self.server.accept()
            except socket.timeout:
                continue
            except OSError:  # the listening socket was closed by stop()
                break
            conn.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            t = threading.Thread(target=self._guarded_session, args=(conn,), daemon=True)
            t.start()
            self.threads.append(t)

    def stop(self):
        self._stop.set()
        self.server.close()

    def _guarded_session(self, conn: socket.socket):
        try:
            self._session(conn)
        except Exception:  # noqa: BLE001 - a failed session ends its connection, not the daemon
            conn.close()

    ENV_KEYS = ("CUDA_VISIBLE_DEVICES",)
    ENV_PREFIXES = ("NCCL_", "DITSERVE_")

    def _session(self, conn: socket.socket):
        first = recv_frame(conn)
        if not first or first.get("bridge") != "spawn":
            conn.close()
            return
        if self.token and not hmac.compare_digest(str(first.get("token", "")), self.token):
            conn.close()
            return
        sdir = os.path.realpath(tempfile.mkdtemp(prefix="session-", dir=self.workdir))
        env = dict(os.environ)
        for k, v in (first.get("env") or {}).items():
            if k in self.ENV_KEYS or k.startswith(self.ENV_PREFIXES):
                env[str(k)] = str(v)
        root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        env["PYTHONPATH"] = root + os.pathsep + env.get("PYTHONPATH", "")
        config = dict(first.get("config", {}))
        # the remote worker always stages packets in its session directory: a client-chosen
        # transfer_dir would widen the file frames' reach (get_file with unlink) to anything
        # the daemon can touch, so the client's value is replaced, never trusted
        config["transfer_dir"] = sdir
        roots = {sdir}
        proc = subprocess.Popen([self.python, "-m", "ditserve_b200.runtime.worker", "--backend", first["backend"],
                                 "--config", json.dumps(config)], stdin=subprocess.PIPE,
                                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True, env=env)
        bells: dict = {}
        send_lock = threading.Lock()

        def reply(obj):
            with send_lock:
                send_frame(conn, obj)

        def confined(path: str) -> str:
            real = os.path.realpath(path)
            if not any(real == r or real.startswith(r + os.sep) for r in roots):
                raise PermissionError(f"{path} is outside the session's directories")
            return real

        def pump():
            for line in proc.stdout:
                reply({"line": line})
        threading.Thread(target=pump, daemon=True).start()
        try:
            while True:
                msg = recv_frame(conn)
                if msg is None:
                    break
                kind = msg.get("bridge")
                if kind is None:
                    proc.stdin.write(msg["line"])
                    proc.stdin.flush()
                elif kind == "ring":
                    slot = str(msg["slot"])
                    if slot not in bells:
                        bells[slot] = Doorbell(os.path.join(sdir, f"bell-{slot}"), create=True)
                    bells[slot].ring(int(msg["epoch"]))
                elif kind == "bell_path":
                    slot = str(msg["slot"])
                    if slot not in bells:
                        bells[slot] = Doorbell(os.path.join(sdir, f"bell-{slot}"), create=True)
                    reply({"bridge": "bell_path", "path": bells[slot].path})
                elif kind == "put_file":
                    try:
                        name = str(msg["name"])
                        if not name or os.path.basename(name) != name or name in (".", ".."):
                            raise PermissionError("put_file takes a plain file name")
                        path = os.path.join(sdir, name)
                        with open(path, "r+b" if int(msg.get("offset", 0)) else "wb") as f:
                            f.seek(int(msg.get("offset", 0)))
                            f.write(base64.b64decode(msg["data_b64"]))
                        reply({"bridge": "put_file", "path": path})
                    except (OSError, ValueError, KeyError) as exc:
                        reply({"bridge": "put_file", "error": str(exc)})
                elif kind == "get_file":
                    try:
                        path = confined(msg["path"])
                        off = int(msg.get("offset", 0))
                        with open(path, "rb") as f:
                            f.seek(off)
                            data = f.read(CHUNK)
                            eof = f.tell() >= os.fstat(f.fileno()).st_size
                        if eof and msg.get("unlink"):
                            os.unlink(path)
                        reply({"bridge": "file", "path": msg["path"], "offset": off,
                               "data_b64": base64.b64encode(data).decode(), "eof": eof})
                    except (OSError, ValueError, KeyError) as exc:
                        reply({"bridge": "file", "path": msg.get("path"), "error": str(exc)})
                elif kind == "occupancy":
                    from .occupancy import occupancy
                    own = [proc.pid] + [int(p) for p in msg.get("own_pids", [])]  # this session's worker is ours
                    reply({"bridge": "occupancy", "result": occupancy(msg.get("gpus"), own_pids=own)})
        finally:
            try:
                proc.stdin.close()
            except OSError:
                pass
            try:
                proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                proc.kill()
            for b in bells.values():
                b.close()
            conn.close()
            shutil.rmtree(sdir, ignore_errors=True)


class BridgeProxy:
    """Stand-in worker: protocol lines on stdin/stdout, relayed to a remote daemon."""

    def __init__(self, address: str, backend: str, config: dict, env: dict | None = None,
                 stage_dir: str | None = None, token: str | None = None):
        host, port = address.rsplit(":", 1)
        self.sock = socket.create_connection((host, int(port)))
        self.sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        token = token if token is not None else os.environ.get("DITSERVE_BRIDGE_TOKEN", "")
        send_frame(self.sock, {"bridge": "spawn", "backend": backend, "config": config, "env": env or {},
                               "token": token})
        shm = "/dev/shm" if os.path.isdir("/dev/shm") else None
        self._own_stage = stage_dir is None
        self.stage_dir = stage_dir or tempfile.mkdtemp(prefix="ds-bridge-stage-", dir=shm)
        self.staged = 0
        self.watch: dict = {}   # local bell path -> (slot, last epoch)
        self.remote_path: dict = {}
        self.lock = threading.Lock()
        self.replies: list = []
        self.cv = threading.Condition()
        self._stop = threading.Event()
        threading.Thread(target=self._reader, daemon=True).start()
        threading.Thread(target=self._watcher, daemon=True).start()

    def _reader(self):
        while True:
            msg = recv_frame(self.sock)
            if msg is None:
                with self.cv:
                    self.replies.append(None)
                    self.cv.notify_all()
                return
            with self.cv:
                self.replies.append(msg)
                self.cv.notify_all()

    def _next(self, pred, timeout=60.0):
        end = time.monotonic() + timeout
        with self.cv:
            while True:
                for i, m in enumerate(self.replies):
                    if m is None or pred(m):
                        return self.replies.pop(i)
                left = end - time.monotonic()
                if left <= 0:
                    raise TimeoutError("bridge reply timed out")
                self.cv.wait(left)

    def _watcher(self):
        while not self._stop.is_set():
            with self.lock:
                items = list(self.watch.items())
            for path, (slot, last) in items:
                try:
                    ep = Doorbell(path).epoch()
                except OSError:
                    continue
                if ep != last:
                    with self.lock:
                        self.watch[path] = (slot, ep)
                        send_frame(self.sock, {"bridge": "ring", "slot": slot, "epoch": ep})
            time.sleep(0.002)

    def _mirror(self, req: dict) -> dict:
        bell = req.get("doorbell")
        if not bell:
            return req
        path = bell["path"]
        with self.lock:
            if path not in self.watch:
                slot = len(self.watch)
                ep = Doorbell(path).epoch()
                self.watch[path] = (slot, ep)
                send_frame(self.sock, {"bridge": "ring", "slot": slot, "epoch": ep})
                send_frame(self.sock, {"bridge": "bell_path", "slot": slot})
                rp = self._next(lambda m: m.get("bridge") == "bell_path")
                self.remote_path[path] = rp["path"]
        return dict(req, doorbell=dict(bell, path=self.remote_path[path]))

    def _call(self, frame: dict, kind: str) -> dict:
        with self.lock:
            send_frame(self.sock, frame)
        msg = self._next(lambda m: m.get("bridge") == kind)
        if msg is None:
            raise ConnectionError("bridge daemon closed the connection")
        if "error" in msg:
            raise OSError(f"bridge {kind}: {msg['error']}")
        return msg

    def push_file(self, local: str) -> str:
        """Copy a local file into the remote session directory; returns the remote path."""
        self.staged += 1
        name = f"in-{self.staged}-{os.path.basename(local)}"
        remote = None
        with open(local, "rb") as f:
            off = 0
            while True:
                data = f.read(CHUNK)
                if off and not data:
                    break
                remote = self._call({"bridge": "put_file", "name": name, "offset": off,
                                     "data_b64": base64.b64encode(data).decode()}, "put_file")["path"]
                off += len(data)
                if len(data) < CHUNK:
                    break
        return remote

    def pull_file(self, remote: str, unlink: bool = True) -> str:
        """Fetch a remote session file into the staging directory; returns the local path."""
        self.staged += 1
        local = os.path.join(self.stage_dir, f"out-{self.staged}-{os.path.basename(remote)}")
        with open(local, "wb") as f:
            off = 0
            while True:
                msg = self._call({"bridge": "get_file", "path": remote, "offset": off, "unlink": unlink}, "file")
                data = base64.b64decode(msg["data_b64"])
                f.write(data)
                off += len(data)
                if msg["eof"]:
                    break
        return local

    def relay(self, line: str) -> str:
        req = None
        pushed = None
        try:
            req = json.loads(line)
            if isinstance(req, dict) and req.get("op") == "bridge_occupancy":
                # answered by the daemon's node, not by the remote worker
                res = self._call({"bridge": "occupancy", "gpus": req.get("gpus"),
                                  "own_pids": req.get("own_pids", [])}, "occupancy")["result"]
                return json.dumps({"version": req.get("version", 1), "id": req.get("id"), "ok": True,
                                   "result": res}) + "\n"
            if isinstance(req, dict):
                req = self._mirror(req)
                if req.get("op") == "block_import" and isinstance(req.get("path"), str) \
                        and os.path.isfile(req["path"]):
                    pushed = req["path"]
                    req = dict(req, path=self.push_file(pushed))
                line = json.dumps(req) + "\n"
        except ValueError:
            pass  # the remote worker produces the protocol error reply
        with self.lock:
            send_frame(self.sock, {"line": line})
        msg = self._next(lambda m: "line" in m)
        if msg is None:
            raise ConnectionError("bridge daemon closed the connection")
        out = msg["line"]
        if isinstance(req, dict) and req.get("op") in ("block_import", "block_export"):
            rep = json.loads(out)
            if rep.get("ok") and pushed is not None:
                os.unlink(pushed)  # consumed, as a local import consumes its packet
            res = rep.get("result")
            if rep.get("ok") and req["op"] == "block_export" and isinstance(res, dict) \
                    and isinstance(res.get("path"), str):
                res["path"] = self.pull_file(res["path"])
                out = json.dumps(rep) + "\n"
        return out

    def close(self):
        self._stop.set()
        self.sock.close()
        if self._own_stage and not os.listdir(self.stage_dir):
            os.rmdir(self.stage_dir)


def main(argv=None):
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="mode", required=True)
    d = sub.add_parser("daemon")
    d.add_argument("--listen", default="127.0.0.1:7700")
    d.add_argument("--token", default=None, help="shared secret (default: DITSERVE_BRIDGE_TOKEN)")
    d.add_argument("--workdir", default=None, help="root of the per-session directories (default: a temp dir)")
    p = sub.add_parser("proxy")
    p.add_argument("--connect", default=os.environ.get("DITSERVE_REMOTE_ENDPOINT"),
                   help="daemon host:port (default: DITSERVE_REMOTE_ENDPOINT)")
    p.add_argument("--backend", required=True)
    p.add_argument("--config", default="{}")
    p.add_argument("--env", action="append", default=[], metavar="KEY=VALUE",
                   help="environment of the remote worker (CUDA_VISIBLE_DEVICES, NCCL_*, DITSERVE_*)")
    p.add_argument("--stage-dir", default=None, help="local directory for packets fetched from the node")
    p.add_argument("--token", default=None, help="shared secret (default: DITSERVE_BRIDGE_TOKEN)")
    args = ap.parse_args(argv)
    if args.mode == "daemon":
        host, port = args.listen.rsplit(":", 1)
        daemon = BridgeDaemon(host, int(port), workdir=args.workdir, token=args.token)
        print(json.dumps({"listening": daemon.port}), flush=True)
        daemon.serve_forever()
        return 0
    if not args.connect:
        ap.error("proxy needs --connect or DITSERVE_REMOTE_ENDPOINT")
    env = dict(kv.split("=", 1) for kv in args.env)
    proxy = BridgeProxy(args.connect, args.backend, json.loads(args.config), env, args.stage_dir, args.token)
    out = sys.stdout
    for line in sys.stdin:
        if not line.strip():
            continue
        out.write(proxy.relay(line))
        out.flush()
    proxy.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
