"""Fixed P/D pairs on CPU worker processes: the router picks a pair per request, each pair's
workers run prefill then decode, and the tokens equal the monolithic engine's; the three
routing policies run side by side on the same requests."""
import torch

from nanovllm_self_b200 import LLM, SamplingParams
from nanovllm_self_b200.pd.multiprocess.audit import audit
from nanovllm_self_b200.pd.multiprocess.pairs import PDPairs, compare_policies, synthetic_rows

ARGS = ["--dtype", "fp32", "--block-size", "16", "--num-blocks", "64", "--max-model-len", "256",
        "--max-num-seqs", "8", "--poll-s", "0.001"]


def _rows():
    g = torch.Generator().manual_seed(17)
    return [{"id": f"q{i}", "prompt_ids": torch.randint(0, 1024, (n,), generator=g).tolist(), "max_tokens": m,
             "input_tokens": n, "session_id": f"s{i % 3}"} for i, (n, m) in
            enumerate([(12, 5), (40, 3), (7, 2), (33, 6), (25, 4), (18, 3)])]


def test_pairs_route_and_match_monolithic(tmp_path):
    rows = _rows()
    ref = LLM("tiny", device="cpu", dtype="fp32", block_size=16, num_blocks=64, max_model_len=256)
    want = {r["id"]: ref.generate([r["prompt_ids"]], SamplingParams(temperature=0, max_tokens=r["max_tokens"],
                                                                    ignore_eos=True))[0][len(r["prompt_ids"]):]
            for r in rows}
    pairs = PDPairs(tmp_path, 2, "shared_memory", "tiny", devices=[("cpu", "cpu")] * 2, worker_args=ARGS,
                    handshake_timeout_s=60)
    pairs.start()
    try:
        res = compare_policies(pairs, rows, concurrency=3, timeout_s=300, warmup=1)
    finally:
        pairs.shutdown()
    assert [r["policy"] for r in res] == ["round_robin", "load_aware", "affinity_load_aware"]
    for summary in res:
        assert summary["num_errors"] == 0 and summary["num_requests"] == len(rows) - 1
        assert sum(summary["requests_per_pair"]) == len(rows) - 1
    assert res[0]["requests_per_pair"][0] > 0 and res[0]["requests_per_pair"][1] > 0  # round robin spreads
    assert res[2]["affinity_hit_rate"] > 0
    # the last run's outputs equal the monolithic engine's
    got = {r["request_id"]: r["output_ids"] for r in pairs.rows_out}
    assert got == {k: v for k, v in want.items() if k in got}
    assert not audit(tmp_path)["processes"]


def test_synthetic_rows_shapes():
    rows = synthetic_rows(50, input_mean=64, output_mean=8, sessions=4, seed=1, vocab=1000, max_input=200)
    assert len(rows) == 50 and all(16 <= r["input_tokens"] <= 200 for r in rows)
    assert all(len(r["prompt_ids"]) == r["input_tokens"] for r in rows)
    assert {r["session_id"] for r in rows} == {"s0", "s1", "s2", "s3"}
