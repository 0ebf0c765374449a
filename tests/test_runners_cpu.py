"""CPU runs of the benchmark drivers that mirror the reference's comparison scripts (tiny model)."""
import json

from nanovllm_self_b200.benchmarks import runners

BASE = ["--model", "tiny", "--device", "cpu", "--max-model-len", "512", "--max-num-seqs", "8", "--block-size", "16"]


def _run(capsys, argv):
    runners.main(argv)
    return json.loads(capsys.readouterr().out.strip().splitlines()[-1])


def test_graph_matrix_reports_every_batch(capsys):
    r = _run(capsys, ["graph_matrix", *BASE, "--batches", "1,3", "--prompt-len", "8", "--gen", "4"])
    assert [p["batch"] for p in r["points"]] == [1, 3]
    assert r["points"][0]["bucket_kind"] == "exact" and r["points"][1]["bucket"] == 4
    for p in r["points"]:
        for mode in ("graph", "eager"):
            assert p[mode]["decode_step_ms"] >= 0 and p[mode]["prefix_hit_blocks_timed"] == 0


def test_mixed_matches_the_oracle_and_reuses_the_prefix(capsys):
    r = _run(capsys, ["mixed", *BASE, "--gen", "6"])
    cases = {x["case"] for x in r["results"]}
    assert cases == {"single_short", "mixed_pair", "batch8_short", "shared_prefix"}
    for x in r["results"]:
        assert all(row["match"] for row in x["rows"]), x
    pre = next(x for x in r["results"] if x["case"] == "shared_prefix")
    assert pre["prefix_hit_blocks"] == pre["expected_hit_blocks"] == 4


def test_decode_vs_hf_on_one_checkpoint(capsys, tmp_path):
    r = _run(capsys, ["decode_vs_hf", *BASE, "--batch", "2", "--prompt-len", "8", "--gen", "4",
                      "--checkpoint", str(tmp_path / "ckpt")])
    assert r["ours_tok_s"] > 0 and r["hf_tok_s"] > 0
    assert 0.0 <= r["first_token_agreement"] <= 1.0
    assert 0 <= r["mean_agreeing_prefix_tokens"] <= 4


def test_prefill_matrix_reports_every_case(capsys):
    r = _run(capsys, ["prefill_matrix", *BASE, "--prompt-lens", "8,40", "--prefill-batches", "1,3", "--gen", "3"])
    assert r["baseline"] == "torch_graph_off"
    assert sorted((c["prompt_len"], c["batch"]) for c in r["cases"]) == [(8, 1), (8, 3), (40, 1), (40, 3)]
    for c in r["cases"]:
        m = c["combos"]["torch_graph_off"]
        assert m["ttft_ms"] > 0 and m["prefill_tok_s"] > 0 and m["decode_tok_s"] > 0
        assert m["prefix_hit_blocks_timed"] == 0
        assert c["gain_vs_torch_graph_off"] == {}
