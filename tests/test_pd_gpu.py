"""P/D on GPUs: in-process coordinator on one GPU, and worker processes on two GPUs moving
the KV with the NVLink IPC push kernel and with NCCL point-to-point.

Every engine here runs in deterministic mode (GEMM plans from the shape alone, so every
process computes a shape with the same kernels) and the pools serve one request at a time (the
decode batch matches the monolithic engine's), so P/D must reproduce the monolithic greedy
tokens exactly."""

import pytest
import torch

from nanovllm_self_b200 import LLM, SamplingParams

pytestmark = pytest.mark.gpu

KW = dict(max_model_len=1024, max_num_seqs=16, num_blocks=128, block_size=16, cuda_graph_max_bs=16,
          deterministic=True)


@pytest.fixture(autouse=True)
def _deterministic_workers(monkeypatch):
    monkeypatch.setenv("NVB_DETERMINISTIC", "1")  # inherited by the worker processes
    yield
    from nanovllm_self_b200.ops._ext import load
    load().gemm_set_deterministic(False)


def _rows():
    g = torch.Generator().manual_seed(31)
    return [{"id": f"q{i}", "prompt_ids": torch.randint(0, 2048, (n,), generator=g).tolist(), "max_tokens": m,
             "input_tokens": n, "session_id": f"s{i % 2}"} for i, (n, m) in enumerate([(40, 8), (150, 12), (9, 1),
                                                                                         (333, 6)])]


def _want():
    llm = LLM("tiny-gpu", device="cuda:0", **KW)
    return {r["id"]: llm.generate([r["prompt_ids"]], SamplingParams(temperature=0, max_tokens=r["max_tokens"],
                                                                     ignore_eos=True))[0][len(r["prompt_ids"]):]
            for r in _rows()}


def _exact(got, want):
    assert got == want, {k: (got.get(k), want[k]) for k in want if got.get(k) != want[k]}


def test_pd_coordinator_single_gpu():
    from nanovllm_self_b200.config import EngineConfig
    from nanovllm_self_b200.pd.coordinator import PDCoordinator
    want = _want()
    pd = PDCoordinator(EngineConfig(model="tiny-gpu", device="cuda:0", **KW))
    rows = _rows()
    got = {}
    for r in rows:
        got[r["id"]] = pd.generate([r["prompt_ids"]], max_tokens=r["max_tokens"])[0][len(r["prompt_ids"]):]
    _exact(got, want)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("backend", ["ipc_push", "sync_gpu"])
def test_pd_pool_two_gpus(tmp_path, backend):
    from nanovllm_self_b200.pd.multiprocess.pool import PDPool
    want = _want()
    args = ["--max-model-len", "1024", "--block-size", "16", "--num-blocks", "128", "--max-num-seqs", "16"]
    pool = PDPool(tmp_path, 1, 1, backend, "tiny-gpu", prefill_devices=["cuda:0"], decode_devices=["cuda:1"],
                  worker_args=args, handshake_timeout_s=60, nccl_port=29731)
    pool.start()
    try:
        s = pool.run(_rows(), concurrency=1, timeout_s=300)
    finally:
        pool.shutdown()
    assert s["num_errors"] == 0, pool.results
    assert pool.exit_codes == [0, 0], pool.exit_codes  # both workers shut down cleanly
    got = {pool.submitted[b]["row"]["id"]: r["output_ids"] for b, r in pool.results.items()}
    _exact(got, want)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_pd_pool_ipc_push_fp8_kv(tmp_path):
    # fp8 KV: the push kernel moves the e4m3 blocks and their per-block scales (which live in
    # the same exported allocation); decode must agree with a monolithic fp8 engine
    from nanovllm_self_b200.pd.multiprocess.pool import PDPool
    llm = LLM("tiny-gpu", device="cuda:0", kv_cache_quant_mode="fp8", **KW)
    want = {r["id"]: llm.generate([r["prompt_ids"]], SamplingParams(temperature=0, max_tokens=r["max_tokens"],
                                                                     ignore_eos=True))[0][len(r["prompt_ids"]):]
            for r in _rows()}
    args = ["--max-model-len", "1024", "--block-size", "16", "--num-blocks", "128", "--max-num-seqs", "16",
            "--kv-cache-quant-mode", "fp8"]
    pool = PDPool(tmp_path, 1, 1, "ipc_push", "tiny-gpu", prefill_devices=["cuda:0"], decode_devices=["cuda:1"],
                  worker_args=args, handshake_timeout_s=60, nccl_port=29761)
    pool.start()
    try:
        s = pool.run(_rows(), concurrency=1, timeout_s=300)
    finally:
        pool.shutdown()
    assert s["num_errors"] == 0, pool.results
    assert pool.exit_codes == [0, 0], pool.exit_codes  # both workers shut down cleanly
    got = {pool.submitted[b]["row"]["id"]: r["output_ids"] for b, r in pool.results.items()}
    _exact(got, want)
