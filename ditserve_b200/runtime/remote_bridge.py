"""Multi-node bridge: a worker on another node behind a local stand-in process.

    # node 1 (the GPUs): serve workers over TCP
    python -m ditserve_b200.runtime.remote_bridge daemon --listen 0.0.0.0:7700
    # node 0 (controller): a process that speaks the worker protocol on stdin/stdout
    python -m ditserve_b200.runtime.remote_bridge proxy --connect node1:7700 --backend wan --config '{...}'

Framing on the wire: 4-byte big-endian length + one JSON document, TCP_NODELAY.
The first frame of a connection is {"bridge": "spawn", "backend", "config"}; the
daemon starts a local worker and relays protocol lines both ways.  Extra frames:
* {"bridge": "ring", "slot", "epoch"} — doorbell mirroring: the proxy watches the
  controller's local doorbell files and the daemon writes the epoch into its own
  copy, so a remote block quantum stops at its next check like a local one;
* {"bridge": "put_file", "path", "data_b64"} / {"bridge": "get_file", "path"} —
  /dev/shm slabs and artifacts;
* {"bridge": "occupancy"} — the remote node's GPU occupancy probe.
Requests naming a doorbell get the path rewritten to the daemon-side mirror.
Reference: workers/ditserve/runtime/remote_bridge.py:1-1009.
"""
from __future__ import annotations

import argparse
import base64
import json
import os
import socket
import struct
import subprocess
import sys
import tempfile
import threading
import time

from .doorbell import Doorbell


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

    def __init__(self, host: str = "127.0.0.1", port: int = 0, python: str = sys.executable, workdir: str | None = None):
        self.server = socket.create_server((host, port))
        self.port = self.server.getsockname()[1]
        self.python = python
        self.workdir = workdir or tempfile.mkdtemp(prefix="ds-bridge-")
        self.threads = []
        self._stop = threading.Event()

    def serve_forever(self):
        self.server.settimeout(0.2)
        while not self._stop.is_set():
            try:
                conn, _ = self.server.accept()
            except socket.timeout:
                continue
            conn.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            t = threading.Thread(target=self._session, args=(conn,), daemon=True)
            t.start()
            self.threads.append(t)

    def stop(self):
        self._stop.set()
        self.server.close()

    def _session(self, conn: socket.socket):
        first = recv_frame(conn)
        if not first or first.get("bridge") != "spawn":
            conn.close()
            return
        env = dict(os.environ)
        root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        env["PYTHONPATH"] = root + os.pathsep + env.get("PYTHONPATH", "")
        proc = subprocess.Popen([self.python, "-m", "ditserve_b200.runtime.worker", "--backend", first["backend"],
                                 "--config", json.dumps(first.get("config", {}))], stdin=subprocess.PIPE,
                                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True, env=env)
        bells: dict = {}
        send_lock = threading.Lock()

        def pump():
            for line in proc.stdout:
                with send_lock:
                    send_frame(conn, {"line": line})
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
                        bells[slot] = Doorbell(os.path.join(self.workdir, f"bell-{slot}"), create=True)
                    bells[slot].ring(int(msg["epoch"]))
                elif kind == "bell_path":
                    slot = str(msg["slot"])
                    if slot not in bells:
                        bells[slot] = Doorbell(os.path.join(self.workdir, f"bell-{slot}"), create=True)
                    with send_lock:
                        send_frame(conn, {"bridge": "bell_path", "path": bells[slot].path})
                elif kind == "put_file":
                    with open(msg["path"], "wb") as f:
                        f.write(base64.b64decode(msg["data_b64"]))
                elif kind == "get_file":
                    with open(msg["path"], "rb") as f:
                        data = base64.b64encode(f.read()).decode()
                    with send_lock:
                        send_frame(conn, {"bridge": "file", "path": msg["path"], "data_b64": data})
                elif kind == "occupancy":
                    from .occupancy import occupancy
                    with send_lock:
                        send_frame(conn, {"bridge": "occupancy", "result": occupancy(msg.get("gpus"))})
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


class BridgeProxy:
    """Stand-in worker: protocol lines on stdin/stdout, relayed to a remote daemon."""

    def __init__(self, address: str, backend: str, config: dict):
        host, port = address.rsplit(":", 1)
        self.sock = socket.create_connection((host, int(port)))
        self.sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        send_frame(self.sock, {"bridge": "spawn", "backend": backend, "config": config})
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

    def relay(self, line: str) -> str:
        try:
            req = json.loads(line)
            if isinstance(req, dict):
                line = json.dumps(self._mirror(req)) + "\n"
        except ValueError:
            pass  # the remote worker produces the protocol error reply
        with self.lock:
            send_frame(self.sock, {"line": line})
        msg = self._next(lambda m: "line" in m)
        if msg is None:
            raise ConnectionError("bridge daemon closed the connection")
        return msg["line"]

    def close(self):
        self._stop.set()
        self.sock.close()


def main(argv=None):
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="mode", required=True)
    d = sub.add_parser("daemon")
    d.add_argument("--listen", default="127.0.0.1:7700")
    p = sub.add_parser("proxy")
    p.add_argument("--connect", required=True)
    p.add_argument("--backend", required=True)
    p.add_argument("--config", default="{}")
    args = ap.parse_args(argv)
    if args.mode == "daemon":
        host, port = args.listen.rsplit(":", 1)
        daemon = BridgeDaemon(host, int(port))
        print(json.dumps({"listening": daemon.port}), flush=True)
        daemon.serve_forever()
        return 0
    proxy = BridgeProxy(args.connect, args.backend, json.loads(args.config))
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
