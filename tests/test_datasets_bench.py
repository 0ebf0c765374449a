"""Workload generators and the configuration search loop (CPU)."""
from nanovllm_self_b200.benchmarks import datasets
from nanovllm_self_b200.benchmarks.optimization import BenchmarkRunner, OptimizationCandidate, OptimizationLoop, \
    TrafficGenerator


def test_generators_are_seeded_and_shaped():
    a = datasets.uniform_serving(8, 1000, (10, 20), (5, 6), seed=1)
    b = datasets.uniform_serving(8, 1000, (10, 20), (5, 6), seed=1)
    assert a == b and all(10 <= r["input_tokens"] <= 20 and 5 <= r["max_tokens"] <= 6 for r in a)
    m = datasets.length_matrix(2, 1000)
    assert len(m) == 2 * len(datasets.PROFILES)
    s = datasets.agent_sessions(3, 1000, prefix_len=64, turns=3, append_mean=16, output_tokens=4)
    assert len(s) == 9
    by = [r for r in s if r["session_id"] == "sess-0"]
    assert by[1]["prompt_ids"][:len(by[0]["prompt_ids"])] == by[0]["prompt_ids"]  # turns extend the context
    assert all(r["prompt_ids"][:64] == s[0]["prompt_ids"][:64] for r in s)  # shared system prefix
    pd = datasets.pd_lognormal(50)
    assert all(16 <= r["input_tokens"] <= 8192 and 4 <= r["max_tokens"] <= 1024 for r in pd)
    assert datasets.classify(2000, 300) == "long_long"


def test_sharegpt_first_turns(tmp_path):
    import json
    p = tmp_path / "sg.json"
    p.write_text(json.dumps([{"id": "c1", "conversations": [{"from": "human", "value": "hi there"},
                                                            {"from": "gpt", "value": "yo"}]}]))
    rows = datasets.sharegpt_first_turns(str(p), lambda t: list(t.encode()))
    assert rows[0]["input_tokens"] == len("hi there")


def test_optimization_loop_picks_a_candidate():
    base = dict(device="cpu", dtype="fp32", block_size=16, num_blocks=128, max_model_len=512)
    loop = OptimizationLoop(BenchmarkRunner("tiny", base), TrafficGenerator(n=4, in_range=(8, 16), out_range=(4, 6)),
                            [OptimizationCandidate("default"),
                             OptimizationCandidate("chunked", {"enable_chunked_prefill": True,
                                                               "prefill_chunk_size": 8})])
    res = loop.run()
    assert res["best"]["candidate"] in ("default", "chunked") and len(res["results"]) == 2


def test_dataset_cli_writes_rows_and_summary(tmp_path, capsys):
    import json
    out = str(tmp_path / "synth.jsonl")
    s = datasets.main(["synthetic", "--per-profile", "3", "--vocab", "1000", "--out", out])
    rows = [json.loads(x) for x in open(out)]
    assert len(rows) == s["rows"] == 3 * len(datasets.PROFILES)
    assert s["rows_per_profile"] == {p: 3 for p in datasets.PROFILES}
    assert s["input_tokens"] == sum(len(r["prompt_ids"]) for r in rows)
    assert json.load(open(out + ".summary.json"))["kind"] == "synthetic"
    a = datasets.main(["agent", "--sessions", "2", "--turns", "3", "--prefix-len", "32", "--vocab", "500",
                       "--out", str(tmp_path / "agent.jsonl")])
    assert a["rows"] == 6 and a["rows_per_session_id"] == {"sess-0": 3, "sess-1": 3}
    capsys.readouterr()
