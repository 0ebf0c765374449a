"""Single-engine baseline, single-vs-P/D comparison and per-request correctness check, on CPU.

The single-engine driver must generate what ``generate`` does for every request under both
arrival processes; a multiprocess P/D pool run (shared-memory KV handoff) must pass the
correctness check against it, through the command line too; and the check must report a
changed token, a missing request and an error row.
"""
import json

import pytest
import torch

from nanovllm_self_b200 import LLM, SamplingParams
from nanovllm_self_b200.pd.multiprocess import evaluation as ev
from nanovllm_self_b200.pd.multiprocess.pool import PDPool

ARGS = ["--dtype", "fp32", "--block-size", "16", "--num-blocks", "64", "--max-model-len", "256",
        "--max-num-seqs", "8", "--poll-s", "0.001"]


def _rows():
    g = torch.Generator().manual_seed(5)
    return [{"id": f"q{i}", "prompt_ids": torch.randint(0, 1024, (n,), generator=g).tolist(), "max_tokens": m,
             "input_tokens": n, "session_id": f"s{i % 2}"}
            for i, (n, m) in enumerate([(9, 4), (30, 2), (17, 7), (44, 3), (5, 5), (21, 1)])]


def _llm():
    return LLM("tiny", device="cpu", dtype="fp32", block_size=16, num_blocks=64, max_model_len=256)


def _want(rows):
    ref = _llm()
    return {r["id"]: ref.generate([r["prompt_ids"]], SamplingParams(temperature=0, max_tokens=r["max_tokens"],
                                                                    ignore_eos=True))[0][len(r["prompt_ids"]):]
            for r in rows}


@pytest.mark.parametrize("concurrency,rate", [(3, None), (None, 500.0)])
def test_single_engine_rows_equal_generate(concurrency, rate):
    rows = _rows()
    want = _want(rows)
    summary, out = ev.run_single(_llm(), rows, concurrency=concurrency, rate=rate, warmup=1)
    assert summary["num_requests"] == len(rows) - 1 and summary["num_errors"] == 0
    assert summary["output_tok_s"] > 0 and summary["ttft_ms_p50"] > 0
    got = {r["request_id"]: r["output_ids"] for r in out}
    assert got == {k: v for k, v in want.items() if k != "q0"}
    for r in out:
        assert r["output_tokens"] == r["max_tokens"] and r["e2e_s"] >= r["ttft_s"] > 0


def test_pool_passes_correctness_against_single(tmp_path, capsys):
    rows = _rows()
    _, single = ev.run_single(_llm(), rows, concurrency=2)
    pool = PDPool(tmp_path / "pool", 1, 1, "shared_memory", "tiny", prefill_devices=["cpu"], decode_devices=["cpu"],
                  worker_args=ARGS, handshake_timeout_s=60, nccl_port=29861)
    pool.start()
    try:
        warm = [dict(r, id="w-" + r["id"]) for r in rows[:2]]
        pool.warmup(warm)
        pd_summary = pool.run(rows, concurrency=3, timeout_s=300)
    finally:
        pool.shutdown()
    pd_rows = pool.request_rows()
    # the summary covers the measured run only; the warm-up rows are flagged and skipped by the check
    assert pd_summary["num_errors"] == 0 and pd_summary["num_requests"] == len(rows)
    assert len(pd_rows) == len(rows) + 2 and sum(r.get("warmup", False) for r in pd_rows) == 2
    res = ev.check_correctness(single, pd_rows)
    assert res["passed"] and res["num_common"] == len(rows), res
    pd_rows = [r for r in pd_rows if not r.get("warmup")]

    # the same check through the command line, on the rows as files
    a, b = tmp_path / "single.jsonl", tmp_path / "pd.jsonl"
    ev.write_rows(a, single)
    ev.write_rows(b, pd_rows)
    ev.main(["correctness", "--left", str(a), "--right", str(b), "--out", str(tmp_path / "c.json")])
    assert json.loads(capsys.readouterr().out)["passed"]
    assert json.loads((tmp_path / "c.json").read_text())["num_mismatches"] == 0

    # one changed token fails the check with its position
    bad = [dict(r) for r in pd_rows]
    k = next(i for i, r in enumerate(bad) if r["output_tokens"] >= 3)
    bad[k]["output_ids"] = bad[k]["output_ids"][:2] + [bad[k]["output_ids"][2] + 1] + bad[k]["output_ids"][3:]
    ev.write_rows(b, bad)
    with pytest.raises(SystemExit):
        ev.main(["correctness", "--left", str(a), "--right", str(b)])
    res = json.loads(capsys.readouterr().out)
    assert not res["passed"] and res["mismatches"][0]["first_divergence"] == 2


def test_correctness_reports_missing_and_error_rows():
    rows = [{"request_id": f"r{i}", "output_ids": [i, i + 1]} for i in range(4)]
    right = [dict(r) for r in rows[1:]]
    right[0] = {"request_id": "r1", "error": "decode worker 0 exited"}
    res = ev.check_correctness(rows, right)
    assert not res["passed"]
    assert res["missing_right"] == ["r0"] and res["num_missing_left"] == 0
    assert res["errors"] == [{"request_id": "r1", "left": None, "right": "decode worker 0 exited"}]
    assert ev.check_correctness(rows, list(reversed(rows)))["passed"]


def test_compare_summaries_ratios(tmp_path, capsys):
    single = {"num_requests": 8, "num_errors": 0, "ttft_ms_p50": 20.0, "tpot_ms_p50": 5.0, "output_tok_s": 1000.0,
              "e2e_s_p90": 2.0}
    pd = {"num_requests": 8, "num_errors": 0, "ttft_ms_p50": 30.0, "tpot_ms_p50": 4.0, "output_tok_s": 1500.0,
          "e2e_s_p90": 0.0}
    res = ev.compare_summaries(single, pd)
    assert res["ttft_ms_p50_pd_over_single"] == 1.5 and res["tpot_ms_p50_pd_over_single"] == 0.8
    assert res["output_tok_s_pd_over_single"] == 1.5 and res["e2e_s_p90_pd_over_single"] == 0.0
    assert "ttft_ms_p99_pd_over_single" not in res
    (tmp_path / "s.json").write_text(json.dumps(single))
    (tmp_path / "p.json").write_text(json.dumps([pd]))
    ev.main(["compare", "--single", str(tmp_path / "s.json"), "--pd", str(tmp_path / "p.json")])
    assert json.loads(capsys.readouterr().out)["output_tok_s_pd_over_single"] == 1.5


def test_policy_report_against_round_robin(tmp_path, capsys):
    sums = [{"policy": "round_robin", "num_requests": 8, "num_errors": 0, "output_tok_s": 100.0, "ttft_ms_p50": 40.0,
             "ttft_ms_p99": 90.0, "tpot_ms_p50": 5.0, "tpot_ms_p99": 6.0, "e2e_s_p90": 2.0,
             "affinity_hit_rate": 0.25, "requests_per_pair": [4, 4]},
            {"policy": "affinity_load_aware", "num_requests": 8, "num_errors": 0, "output_tok_s": 125.0,
             "ttft_ms_p50": 30.0, "ttft_ms_p99": 70.0, "tpot_ms_p50": 5.0, "tpot_ms_p99": 6.5, "e2e_s_p90": 1.5,
             "affinity_hit_rate": 0.75, "requests_per_pair": [6, 2]}]
    rep = ev.policy_report(sums)
    rr, aff = rep["policies"]
    assert rep["baseline"] == "round_robin" and rr["output_tok_s_over_round_robin"] == 1.0
    assert aff["output_tok_s_over_round_robin"] == 1.25 and aff["ttft_ms_p50_over_round_robin"] == 0.75
    assert rr["pair_imbalance"] == 1.0 and aff["pair_imbalance"] == 1.5
    md = ev.markdown_table(rep)
    assert md.count("\n") == 4 and "| affinity_load_aware | 125.0 | 1.25 |" in md
    (tmp_path / "a.json").write_text(json.dumps(sums[:1]))
    (tmp_path / "b.json").write_text(json.dumps(sums[1]))
    ev.main(["policies", "--summaries", str(tmp_path / "a.json"), str(tmp_path / "b.json"),
             "--markdown", str(tmp_path / "p.md")])
    assert [r["policy"] for r in json.loads(capsys.readouterr().out)["policies"]] == ["round_robin",
                                                                                    "affinity_load_aware"]
    assert (tmp_path / "p.md").read_text() == md


def test_single_runs_a_prepared_dataset(tmp_path, capsys):
    from nanovllm_self_b200.benchmarks import datasets
    from nanovllm_self_b200.pd.multiprocess.pairs import load_rows
    path = str(tmp_path / "u.jsonl")
    datasets.main(["uniform", "--num-requests", "5", "--vocab", "1024", "--out", path])
    rows = load_rows(path, 3)
    assert len(rows) == 3 and all(r["input_tokens"] == len(r["prompt_ids"]) for r in rows)
    capsys.readouterr()
    out = str(tmp_path / "single.json")
    ev.main(["single", "--model", "tiny", "--device", "cpu", "--dtype", "fp32", "--max-model-len", "2048",
             "--block-size", "16", "--dataset", path, "--num-requests", "2", "--warmup", "1", "--concurrency", "2",
             "--out", out])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["num_requests"] == 2 and res["num_errors"] == 0
    assert [r["request_id"] for r in ev.read_rows(out + ".jsonl")] != []
