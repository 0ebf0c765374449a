"""Multiprocess P/D on CPU: persistent prefill and decode worker processes over shared memory.

The handshake files, error files, worker state and shutdown are exercised for real; the
tokens must equal the monolithic engine's.  Also: router policies, control-plane socket
path and failure cases (a malformed request file, a decode worker that never answers).
"""
import json
import time

import pytest
import torch

from nanovllm_self_b200 import LLM, SamplingParams
from nanovllm_self_b200.pd.multiprocess.agent_scheduler import Router, RouterConfig, estimate
from nanovllm_self_b200.pd.multiprocess.control_plane import WorkDir, connect_control, control_socket_path, \
    make_control_listener
from nanovllm_self_b200.pd.multiprocess.pool import PDPool

ARGS = ["--dtype", "fp32", "--block-size", "16", "--num-blocks", "64", "--max-model-len", "256",
        "--max-num-seqs", "8", "--poll-s", "0.001"]


def _rows():
    g = torch.Generator().manual_seed(21)
    return [{"id": f"q{i}", "prompt_ids": torch.randint(0, 1024, (n,), generator=g).tolist(), "max_tokens": m,
             "input_tokens": n, "session_id": f"s{i % 2}"} for i, (n, m) in enumerate([(12, 6), (40, 3), (7, 1), (33, 9)])]


def test_pool_shared_memory_matches_monolithic(tmp_path):
    rows = _rows()
    ref = LLM("tiny", device="cpu", dtype="fp32", block_size=16, num_blocks=64, max_model_len=256)
    want = {r["id"]: ref.generate([r["prompt_ids"]], SamplingParams(temperature=0, max_tokens=r["max_tokens"],
                                                                    ignore_eos=True))[0][len(r["prompt_ids"]):]
            for r in rows}
    pool = PDPool(tmp_path, 1, 1, "shared_memory", "tiny", prefill_devices=["cpu"], decode_devices=["cpu"],
                  policy="affinity_load_aware", worker_args=ARGS, handshake_timeout_s=60)
    pool.start()
    try:
        summary = pool.run(rows, concurrency=2, timeout_s=300)
    finally:
        pool.shutdown()
    assert summary["num_errors"] == 0, pool.results
    got = {pool.submitted[b]["row"]["id"]: r["output_ids"] for b, r in pool.results.items()}
    assert got == want
    assert summary["ttft_ms_p50"] > 0 and summary["output_tok_s"] > 0
    # workers wrote their load files and exited on shutdown
    assert (tmp_path / "prefill_0" / "worker_state.json").exists()


def test_bad_request_file_reports_error_and_worker_survives(tmp_path):
    pool = PDPool(tmp_path, 1, 1, "shared_memory", "tiny", prefill_devices=["cpu"], decode_devices=["cpu"],
                  worker_args=ARGS, handshake_timeout_s=30)
    pool.start()
    try:
        pool.pwd[0].write_json("bad.request.json", {"prompt_ids": "not-a-list", "max_tokens": 3,
                                                    "decode_work_dir": str(pool.dwd[0].path)})
        deadline = time.time() + 60
        while not pool.dwd[0].exists("bad.prefill_error.json") and time.time() < deadline:
            time.sleep(0.05)
        assert pool.dwd[0].exists("bad.prefill_error.json")
        s = pool.run(_rows()[:1], concurrency=1, timeout_s=120)
        assert s["num_errors"] == 0
    finally:
        pool.shutdown()


def test_router_policies():
    cfg = RouterConfig()
    reqs = [estimate({"input_tokens": 100 * (i + 1), "session_id": "a" if i % 2 else "b"}, i, 64, cfg)
            for i in range(6)]
    rr = Router(3, "round_robin")
    assert [rr.route(r, 0.0)["worker_id"] for r in reqs] == [0, 1, 2, 0, 1, 2]
    la = Router(3, "load_aware")
    picks = [la.route(r, 0.0)["worker_id"] for r in reqs]
    assert len(set(picks[:3])) == 3  # spreads while idle
    aff = Router(3, "affinity_load_aware")
    m = [aff.route(r, 0.0) for r in reqs]
    assert any(x["affinity_hit"] for x in m)
    assert estimate({"prompt": "please search the database"}, 0, 10, cfg).task_type == "tool_like"
    with pytest.raises(ValueError):
        Router(2, "nope")


def test_control_socket_roundtrip(tmp_path):
    path = control_socket_path(tmp_path)
    listener = make_control_listener(path)
    import threading
    got = []

    def serve():
        c = listener.accept()
        got.append(c.recv())
        c.send({"ok": True})
        c.close()
    th = threading.Thread(target=serve)
    th.start()
    c = connect_control(path, timeout_s=5)
    c.send({"type": "payload_ready", "base": "r1"})
    assert c.recv() == {"ok": True}
    th.join()
    listener.close()
    assert got == [{"type": "payload_ready", "base": "r1"}]
    assert control_socket_path("/" + "x" * 200).startswith("/tmp/")
    with pytest.raises(TimeoutError):
        connect_control(str(tmp_path / "nobody.sock"), timeout_s=0.2)


def test_pool_tp2_groups_match_monolithic(tmp_path):
    # a prefill group and a decode group, each TP=2 (gloo on CPU, one torchrun per group):
    # rank 0 of each group drives the work directory, the other rank follows in lockstep,
    # and every rank hands its own KV-head shard over shared memory
    rows = _rows()
    ref = LLM("tiny", device="cpu", dtype="fp32", block_size=16, num_blocks=64, max_model_len=256)
    want = {r["id"]: ref.generate([r["prompt_ids"]], SamplingParams(temperature=0, max_tokens=r["max_tokens"],
                                                                    ignore_eos=True))[0][len(r["prompt_ids"]):]
            for r in rows}
    pool = PDPool(tmp_path, 1, 1, "shared_memory", "tiny", worker_args=ARGS, handshake_timeout_s=120, tp=2,
                  device_kind="cpu", nccl_port=29740)
    pool.start(ready_timeout_s=300)
    try:
        summary = pool.run(rows, concurrency=2, timeout_s=300)
    finally:
        pool.shutdown()
    assert summary["num_errors"] == 0, pool.results
    got = {pool.submitted[b]["row"]["id"]: r["output_ids"] for b, r in pool.results.items()}
    assert got == want
    assert json.loads((tmp_path / "decode_0" / "worker_ready.json").read_text())["tp"] == 2


@pytest.mark.parametrize("backend,caps", [("shared_memory", ["--max-active-decode-requests", "1"])])
def test_backpressure_caps_throttle_without_losing_requests(tmp_path, backend, caps):
    """With one admitted decode request at a time, a burst of requests still completes with the
    monolithic engine's tokens: the handoffs beyond the cap wait in the work directory instead of
    failing.  (The NCCL send / receive caps apply to the sync_gpu backend, which runs on GPUs.)"""
    rows = _rows()
    ref = LLM("tiny", device="cpu", dtype="fp32", block_size=16, num_blocks=64, max_model_len=256)
    want = {r["id"]: ref.generate([r["prompt_ids"]], SamplingParams(temperature=0, max_tokens=r["max_tokens"],
                                                                    ignore_eos=True))[0][len(r["prompt_ids"]):]
            for r in rows}
    pool = PDPool(tmp_path, 1, 1, backend, "tiny", prefill_devices=["cpu"], decode_devices=["cpu"],
                  worker_args=ARGS + caps, handshake_timeout_s=60, nccl_port=29841)
    pool.start()
    try:
        summary = pool.run(rows, concurrency=4, timeout_s=300)
    finally:
        pool.shutdown()
    assert summary["num_errors"] == 0, pool.results
    assert pool.exit_codes == [0, 0], pool.exit_codes
    got = {pool.submitted[b]["row"]["id"]: r["output_ids"] for b, r in pool.results.items()}
    assert got == want
