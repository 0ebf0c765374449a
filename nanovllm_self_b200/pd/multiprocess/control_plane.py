"""Control plane between worker processes: AF_UNIX message sockets plus a file protocol.

Reference: ``pd_self/multiprocess/control_plane.py:8-51`` (socket path hashed into /tmp
when too long for AF_UNIX, client connect with retry) and the file protocol of the
persistent workers (``persistent_prefill_worker.py:159-193``).  Only small control
messages travel here; KV data goes through a KV store backend or the IPC push.
"""
from __future__ import annotations

import hashlib
import json
import os
import pickle
import time
from multiprocessing.connection import Client, Listener
from pathlib import Path

SOCKET_NAME = "pd_control.sock"


def control_socket_path(work_dir) -> str:
    p = str(Path(work_dir) / SOCKET_NAME)
    if len(p) < 100:
        return p
    digest = hashlib.sha1(str(work_dir).encode()).hexdigest()[:16]
    return f"/tmp/nvb_pd_{digest}.sock"


def make_control_listener(sock_path: str) -> Listener:
    try:
        os.unlink(sock_path)
    except FileNotFoundError:
        pass
    return Listener(sock_path, family="AF_UNIX")


def connect_control(sock_path: str, timeout_s: float = 120.0, poll_interval_s: float = 0.05):
    deadline = time.time() + timeout_s
    while time.time() < deadline:
        try:
            return Client(sock_path, family="AF_UNIX")
        except (FileNotFoundError, ConnectionRefusedError):
            time.sleep(poll_interval_s)
    raise TimeoutError(f"timed out connecting control socket: {sock_path}")


class WorkDir:
    """File protocol of one worker's directory.

    ``<base>.request.json`` (driver -> prefill), ``<base>.payload.pkl`` (prefill -> decode),
    ``<base>.payload_ready`` / ``<base>.recv_ready`` / ``<base>.push_done`` (handshake),
    ``<base>.prefill_done`` / ``<base>.decode_done`` (completion), ``<base>.<stage>_metrics.json``,
    ``<base>.<stage>_error.json``, ``worker_state.json``, ``worker_ready.json`` and ``shutdown``.
    Every file is written to a temporary name and renamed, so readers never see a torn file.
    """

    def __init__(self, path):
        self.path = Path(path)
        self.path.mkdir(parents=True, exist_ok=True)

    def f(self, name: str) -> Path:
        return self.path / name

    def write_json(self, name: str, obj) -> None:
        tmp = self.f(f".{name}.tmp.{os.getpid()}")
        with open(tmp, "w") as fh:
            json.dump(obj, fh)
        os.replace(tmp, self.f(name))

    def read_json(self, name: str):
        with open(self.f(name)) as fh:
            return json.load(fh)

    def write_pickle(self, name: str, obj) -> None:
        tmp = self.f(f".{name}.tmp.{os.getpid()}")
        with open(tmp, "wb") as fh:
            pickle.dump(obj, fh)
        os.replace(tmp, self.f(name))

    def read_pickle(self, name: str):
        with open(self.f(name), "rb") as fh:
            return pickle.load(fh)

    def touch(self, name: str, content: str = "") -> None:
        self.write_json(name, {"t": time.time(), "msg": content}) if content else self.write_json(name, {"t": time.time()})

    def exists(self, name: str) -> bool:
        return self.f(name).exists()

    def remove(self, name: str) -> None:
        try:
            self.f(name).unlink()
        except FileNotFoundError:
            pass

    def glob(self, pattern: str) -> list:
        return sorted(self.path.glob(pattern), key=lambda p: p.stat().st_mtime if p.exists() else 0)

    def shutdown_requested(self) -> bool:
        return self.exists("shutdown")

    def wait_for(self, name: str, timeout_s: float, poll_s: float = 0.002) -> bool:
        deadline = time.time() + timeout_s
        while time.time() < deadline:
            if self.exists(name):
                return True
            if self.shutdown_requested():
                return False
            time.sleep(poll_s)
        return False
