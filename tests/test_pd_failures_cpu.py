"""Host-side failure cases of the multiprocess P/D pool, on CPU worker processes.

A worker killed in the middle of a request, a truncated payload file, duplicated and lost
control messages, and the post-run resource audit (leftover processes, error files, pending
state, handshake leftovers, sockets, leaked shared-memory segments).  No GPU is involved:
every failure is made on the host.
"""
import os
import pickle
import signal
import time
from pathlib import Path

import pytest
import torch

from nanovllm_self_b200.pd.multiprocess.audit import SHM_DIR, SHM_PREFIX, audit
from nanovllm_self_b200.pd.multiprocess.pool import PDPool

ARGS = ["--dtype", "fp32", "--block-size", "16", "--num-blocks", "64", "--max-model-len", "512",
        "--max-num-seqs", "8", "--poll-s", "0.001"]


def _rows(n=2, max_tokens=6, seed=3):
    g = torch.Generator().manual_seed(seed)
    return [{"id": f"q{i}", "prompt_ids": torch.randint(0, 1024, (20 + 7 * i,), generator=g).tolist(),
             "max_tokens": max_tokens, "input_tokens": 20 + 7 * i} for i in range(n)]


def _pool(tmp_path, timeout_s=30.0):
    return PDPool(tmp_path, 1, 1, "shared_memory", "tiny", prefill_devices=["cpu"], decode_devices=["cpu"],
                  worker_args=ARGS, handshake_timeout_s=timeout_s)


def _wait(pred, timeout_s=60.0):
    deadline = time.time() + timeout_s
    while time.time() < deadline:
        if pred():
            return True
        time.sleep(0.01)
    return False


def _our_shm():
    return {p.name for p in SHM_DIR.glob(f"{SHM_PREFIX}*")} if SHM_DIR.exists() else set()


def _unlink_shm(names):
    for n in names:
        try:
            (SHM_DIR / n).unlink()
        except FileNotFoundError:
            pass


def test_clean_run_passes_the_audit(tmp_path):
    before = _our_shm()
    pool = _pool(tmp_path)
    pool.start()
    try:
        s = pool.run(_rows(), concurrency=2, timeout_s=120)
        assert s["num_errors"] == 0, pool.results
    finally:
        pool.shutdown()
    assert all(c == 0 for c in pool.exit_codes), pool.exit_codes  # every worker shut down cleanly
    rep = audit(tmp_path)
    assert not rep["processes"] and not rep["error_files"] and not rep["handshake_leftovers"], rep
    assert not rep["pending_state"] and not rep["sockets"], rep
    assert not (set(rep["shm_segments"]) - before), rep


def test_decode_worker_killed_mid_request(tmp_path):
    """The decode worker dies while decoding: its requests fail fast, the audit sees the debris."""
    before = _our_shm()
    pool = _pool(tmp_path)
    pool.start()
    dwd = pool.dwd[0]
    try:
        row = _rows(1, max_tokens=400)[0]
        base = pool.submit(row, 0, 0.0)
        # the handoff happened: the decode worker is now restoring / decoding this request
        assert _wait(lambda: dwd.exists(f"{base}.prefill_done"), 120)
        time.sleep(0.05)
        assert not dwd.exists(f"{base}.decode_done")
        pool.procs[1].send_signal(signal.SIGKILL)
        pool.procs[1].wait(timeout=30)
        failed = pool._fail_stuck({base}, request_timeout_s=None)
        assert failed == [base] and "decode worker 0 exited" in pool.results[base]["error"]
        # a second request routed to the dead worker fails too instead of stalling the run
        n_before = len(pool.results)
        pool.run(_rows(1, seed=5), concurrency=1, timeout_s=60)
        new = [r for b, r in pool.results.items() if b != base]
        assert len(pool.results) == n_before + 1 and "decode worker 0 exited" in new[0]["error"]
        rep = audit(tmp_path)
        assert [p["pid"] for p in rep["processes"]] == [pool.procs[0].pid]  # the prefill worker lives on
        # both requests' handoffs were left in the dead worker's directory
        left = {Path(p).name for p in rep["handshake_leftovers"]}
        assert {f"{base}.payload.pkl", f"{base}.prefill_done"} <= left, rep
    finally:
        pool.shutdown()
        _unlink_shm(_our_shm() - before)
    rep = audit(tmp_path)
    assert not rep["processes"], rep


def test_truncated_payload_reports_error_and_worker_survives(tmp_path):
    pool = _pool(tmp_path)
    pool.start()
    dwd = pool.dwd[0]
    try:
        blob = pickle.dumps({"not": "a payload", "pad": list(range(1000))})
        (Path(dwd.path) / "trunc.payload.pkl").write_bytes(blob[: len(blob) // 2])
        dwd.touch("trunc.prefill_done")
        assert _wait(lambda: dwd.exists("trunc.decode_error.json"), 60)
        assert "pickle" in dwd.read_json("trunc.decode_error.json")["error"].lower() or \
            "truncat" in dwd.read_json("trunc.decode_error.json")["error"].lower() or \
            "EOF" in dwd.read_json("trunc.decode_error.json")["error"]
        s = pool.run(_rows(1), concurrency=1, timeout_s=120)
        assert s["num_errors"] == 0, pool.results
        rep = audit(tmp_path)
        assert rep["error_files"] == [str(Path(dwd.path) / "trunc.decode_error.json")]
    finally:
        pool.shutdown()


def test_duplicated_control_messages_are_served_once(tmp_path):
    pool = _pool(tmp_path)
    pool.start()
    pwd, dwd = pool.pwd[0], pool.dwd[0]
    try:
        row = _rows(1)[0]
        s = pool.run([row], concurrency=1, timeout_s=120)
        assert s["num_errors"] == 0
        base = next(iter(pool.results))
        first = dwd.read_json(f"{base}.decode_metrics.json")
        mtime = (Path(dwd.path) / f"{base}.decode_done").stat().st_mtime
        # the same request and the same completion marker arrive a second time
        req = {"request_id": row["id"], "prompt_ids": row["prompt_ids"], "max_tokens": row["max_tokens"],
               "decode_work_dir": str(dwd.path)}
        pwd.write_json(f"{base}.request.json", req)
        dwd.touch(f"{base}.prefill_done")
        time.sleep(1.0)
        assert (Path(dwd.path) / f"{base}.decode_done").stat().st_mtime == mtime
        assert dwd.read_json(f"{base}.decode_metrics.json") == first
        assert not list(Path(dwd.path).glob("*_error.json"))
        # both workers still serve
        s = pool.run(_rows(1, seed=9), concurrency=1, timeout_s=120)
        assert s["num_errors"] == 0, pool.results
    finally:
        pool.shutdown()


def test_lost_request_message_times_out_alone(tmp_path):
    pool = _pool(tmp_path)
    pool.start()
    real_write = pool.pwd[0].write_json

    def lossy_write(name, obj):  # the driver's message for request "lost" never arrives
        if name.endswith(".request.json") and obj.get("request_id") == "lost":
            return
        real_write(name, obj)

    pool.pwd[0].write_json = lossy_write
    try:
        rows = _rows(2)
        rows[1]["id"] = "lost"
        s = pool.run(rows, concurrency=2, timeout_s=120, request_timeout_s=10)
        assert s["num_errors"] == 1
        errs = [r for r in pool.results.values() if "error" in r]
        assert "no completion within" in errs[0]["error"]
    finally:
        pool.shutdown()
    assert not audit(tmp_path)["processes"]


@pytest.mark.skipif(not hasattr(os, "kill"), reason="needs POSIX signals")
def test_audit_reports_each_kind_of_leftover(tmp_path):
    wd = tmp_path / "decode_0"
    wd.mkdir()
    import json
    import subprocess
    import sys
    proc = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(60)"])
    try:
        (wd / "worker_ready.json").write_text(json.dumps({"pid": proc.pid}))
        (wd / "worker_state.json").write_text(json.dumps({"busy": True, "pending_push": 2}))
        (wd / "r1.decode_error.json").write_text("{}")
        (wd / "r2.recv_ready").write_text("{}")
        (wd / "r3.payload.pkl").write_text("")
        (wd / "r3.decode_done").write_text("{}")  # completed: not a leftover
        (wd / "pd_control.sock").write_text("")
        rep = audit(tmp_path, shm_dir=tmp_path / "no_shm")
        assert rep["processes"] == [{"dir": str(wd), "pid": proc.pid}]
        assert rep["error_files"] == [str(wd / "r1.decode_error.json")]
        assert rep["pending_state"][0]["pending_push"] == 2
        assert rep["handshake_leftovers"] == [str(wd / "r2.recv_ready")]
        assert rep["sockets"] == [str(wd / "pd_control.sock")]
        assert rep["clean"] is False
    finally:
        proc.kill()
        proc.wait()
    assert not audit(tmp_path, shm_dir=tmp_path / "no_shm")["processes"]


@pytest.mark.skipif(not hasattr(signal, "SIGSTOP"), reason="needs POSIX job-control signals")
def test_stalled_decode_worker_times_out_then_recovers(tmp_path):
    """A decode worker that stops answering (SIGSTOP) makes its request time out alone; once it
    runs again (SIGCONT) it serves new requests and shuts down cleanly."""
    pool = _pool(tmp_path)
    pool.start()
    dproc = pool.procs[1]
    try:
        os.kill(dproc.pid, signal.SIGSTOP)
        try:
            s = pool.run(_rows(1, seed=11), concurrency=1, timeout_s=120, request_timeout_s=5)
        finally:
            os.kill(dproc.pid, signal.SIGCONT)
        assert s["num_errors"] == 1
        assert "no completion within" in next(iter(pool.results.values()))["error"]
        assert dproc.poll() is None  # stalled, not dead
        n_before = len(pool.results)
        s = pool.run(_rows(2, seed=12), concurrency=2, timeout_s=120, request_timeout_s=60)
        new = list(pool.results.values())[n_before:]
        assert len(new) == 2 and all("error" not in r for r in new), new
    finally:
        pool.shutdown()
    assert all(c == 0 for c in pool.exit_codes), pool.exit_codes
    assert not audit(tmp_path)["processes"]
