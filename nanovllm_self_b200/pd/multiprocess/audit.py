"""Post-run resource audit of a P/D worker pool.

Reference: ``pd_self/multiprocess/evaluation/check_pd_resource_cleanup.py:25-150``, which
looks for leftover worker processes, error files, state files that still report pending
work, control sockets and leaked ``/dev/shm`` segments after a run.  Same checks here, over
this package's file protocol:

* ``processes``: pids recorded in each worker's ``worker_ready.json`` that are still alive;
* ``error_files``: ``*_error.json`` files (each is one failed request);
* ``pending_state``: ``worker_state.json`` files whose worker reported work in flight
  (busy, queued requests, pending sends / receives / pushes, active decodes);
* ``handshake_leftovers``: ``payload.pkl`` files and ``prefill_done`` / ``payload_ready`` /
  ``recv_ready`` markers of requests that never completed (no ``decode_done`` and no error
  file), e.g. those handed to a decode worker that died;
* ``sockets``: control sockets left in the work directories (or their hashed ``/tmp`` names);
* ``shm_segments``: ``/dev/shm`` segments of the shared-memory KV store (``nvb_kv_*``).

``audit(work_root)`` returns a dict of those lists plus ``clean`` (all empty);
``python -m nanovllm_self_b200.pd.multiprocess.audit <work_root>`` prints it as JSON and exits
non-zero when something leaked.
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

from .control_plane import SOCKET_NAME, control_socket_path

SHM_DIR = Path("/dev/shm")
SHM_PREFIX = "nvb_kv_"


def _alive(pid: int) -> bool:
    try:
        os.kill(pid, 0)
    except ProcessLookupError:
        return False
    except PermissionError:
        return True
    # a zombie (exited, not reaped) is not a leftover worker
    try:
        with open(f"/proc/{pid}/stat") as f:
            return f.read().split(")")[-1].split()[0] != "Z"
    except OSError:
        return True


def _worker_dirs(root: Path) -> list:
    return sorted(p.parent for p in root.glob("*/worker_ready.json")) or sorted(p for p in root.iterdir() if p.is_dir())


def audit(work_root, shm_dir: Path = SHM_DIR, shm_owner_pids=None) -> dict:
    root = Path(work_root)
    report = {"processes": [], "error_files": [], "pending_state": [], "handshake_leftovers": [], "sockets": [],
              "shm_segments": []}
    if not root.exists():
        report["clean"] = True
        return report
    for wd in _worker_dirs(root):
        ready = wd / "worker_ready.json"
        if ready.exists():
            try:
                pid = int(json.loads(ready.read_text())["pid"])
                if _alive(pid):
                    report["processes"].append({"dir": str(wd), "pid": pid})
            except (ValueError, KeyError, json.JSONDecodeError):
                pass
        report["error_files"] += [str(p) for p in sorted(wd.glob("*_error.json"))]
        st = wd / "worker_state.json"
        if st.exists():
            try:
                s = json.loads(st.read_text())
                pending = {k: s.get(k) for k in ("busy", "queue_depth", "pending_sends", "pending_recvs",
                                                 "pending_push", "active") if s.get(k)}
                if pending:
                    report["pending_state"].append({"file": str(st), **pending})
            except json.JSONDecodeError:
                report["pending_state"].append({"file": str(st), "unreadable": True})
        for marker in ("payload.pkl", "prefill_done", "payload_ready", "recv_ready"):
            for p in sorted(wd.glob(f"*.{marker}")):
                base = p.name[:-len(f".{marker}")]
                finished = (wd / f"{base}.decode_done").exists() or any(wd.glob(f"{base}.*_error.json"))
                if not finished:
                    report["handshake_leftovers"].append(str(p))
        for sock in {str(wd / SOCKET_NAME), control_socket_path(wd)}:
            if os.path.exists(sock):
                report["sockets"].append(sock)
    if shm_dir.exists():
        report["shm_segments"] = sorted(p.name for p in shm_dir.glob(f"{SHM_PREFIX}*"))
    report["clean"] = not any(report[k] for k in report)
    return report


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv:
        print("usage: python -m nanovllm_self_b200.pd.multiprocess.audit <work_root>", file=sys.stderr)
        return 2
    rep = audit(argv[0])
    print(json.dumps(rep, indent=1))
    return 0 if rep["clean"] else 1


if __name__ == "__main__":
    sys.exit(main())
