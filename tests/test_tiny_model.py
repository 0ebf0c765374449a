"""Benchmark config 1: tiny random-init Qwen3 on CPU in fp32, paged KV with block 16.

Greedy tokens from the engine must equal a dense no-cache forward of the same weights
(the reference's HF-equality oracle, ``tests/test_compare_with_hf.py``, re-targeted at
random weights).
"""
import pytest
import torch

from nanovllm_self_b200 import LLM, SamplingParams
from nanovllm_self_b200.models.reference import greedy_generate

LENS = (16, 32, 48, 64)


@pytest.fixture(scope="module")
def prompts():
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, 1024, (n,), generator=g).tolist() for n in LENS]


def _llm(**kw):
    base = dict(device="cpu", dtype="fp32", block_size=16, max_model_len=512, num_blocks=128)
    base.update(kw)
    return LLM("tiny", **base)


def _oracle(llm, prompts, n):
    return [greedy_generate(llm.model_runner.model, p, n) for p in prompts]


def test_config1_greedy_equals_dense_oracle(prompts):
    llm = _llm()
    out = llm.generate(prompts, SamplingParams(temperature=0, max_tokens=32, ignore_eos=True))
    ref = _oracle(llm, prompts, 32)
    for p, o, r in zip(prompts, out, ref):
        assert o[:len(p)] == p
        assert o[len(p):] == r


def test_chunked_prefill_equals_oracle(prompts):
    llm = _llm(enable_chunked_prefill=True, prefill_chunk_size=20, max_num_batched_tokens=40)
    out = llm.generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
    ref = _oracle(llm, prompts, 8)
    for p, o, r in zip(prompts, out, ref):
        assert o[len(p):] == r


def test_prefix_hit_computes_only_suffix(prompts):
    llm = _llm()
    base = prompts[3]
    llm.generate([base], SamplingParams(temperature=0, max_tokens=2, ignore_eos=True))
    longer = base + [5, 6, 7, 8, 9]
    seq = llm.add_request(longer, SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))
    assert seq.num_cached_tokens == 0
    scheduled = llm.scheduler.schedule()
    assert scheduled == [seq]
    assert seq.num_cached_tokens == 64 and seq.num_new_tokens == len(longer) - 64
    need = [0]
    toks, need = llm.model_runner.run(scheduled)
    llm.scheduler.postprocess(scheduled, toks, need)
    while not llm.is_finished():
        llm.step()
    assert seq.completion_token_ids == greedy_generate(llm.model_runner.model, longer, 6)


def test_session_prefix_cache_reuse(prompts):
    llm = _llm()
    sp = SamplingParams(temperature=0, max_tokens=4, ignore_eos=True)
    first = llm.generate([prompts[2]], sp, request_metadata={"session_id": "s1"})[0]
    second_prompt = first + [11, 12, 13]
    seq = llm.add_request(second_prompt, sp, session_id="s1")
    llm.scheduler.schedule()
    assert seq.prefix_cache_source == "session_local" and seq.num_cached_tokens == 48
    llm.scheduler.postprocess([seq], *llm.model_runner.run([seq]))
    while not llm.is_finished():
        llm.step()
    assert seq.completion_token_ids == greedy_generate(llm.model_runner.model, second_prompt, 4)


def test_preemption_keeps_outputs(prompts):
    llm = _llm(num_blocks=10, max_model_len=128)
    out = llm.generate(prompts, SamplingParams(temperature=0, max_tokens=24, ignore_eos=True), return_metrics=True)
    assert out["metrics"]["num_preemptions"] > 0
    ref = _oracle(llm, prompts, 24)
    for p, o, r in zip(prompts, out["outputs"], ref):
        assert o[len(p):] == r


def test_sampling_temperature_and_metrics(prompts):
    llm = _llm()
    out = llm.generate(prompts, [SamplingParams(temperature=1.0, max_tokens=8, ignore_eos=True, top_p=0.9)] * 4,
                       return_metrics=True)
    m = out["metrics"]
    assert m["generated_tokens"] == 32 and m["num_seqs"] == 4
    for o in out["outputs"]:
        assert all(0 <= t < 1024 for t in o)
    assert m["ttft_ms_p50"] > 0


def test_int8_mock_and_fp8_kv_close_to_oracle(prompts):
    for mode in ("int8_mock", "fp8"):
        llm = _llm(kv_cache_quant_mode=mode)
        out = llm.generate(prompts[:2], SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))
        ref = _oracle(llm, prompts[:2], 6)
        agree = sum(a == b for o, r, p in zip(out, ref, prompts) for a, b in zip(o[len(p):], r))
        assert agree >= 10, (mode, agree)


def test_profile_summary_and_nvtx_off(capsys):
    from nanovllm_self_b200 import LLM, SamplingParams
    from nanovllm_self_b200.engine.llm_engine import LLMEngine
    eng = LLMEngine(enable_profile=True, model="tiny", device="cpu", block_size=16, max_model_len=256,
                    dtype="fp32", num_blocks=64)
    res = eng.generate([[1, 2, 3, 4, 5]], SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True),
                       return_metrics=True)
    prof = res["metrics"]["profile"]
    assert prof["steps"] == prof["prefill_steps"] + prof["decode_steps"] and prof["decode_steps"] >= 3
    assert prof["host_run_ms"] > 0
    assert "[PROFILE]" in capsys.readouterr().out


def test_metrics_jsonl_appends_one_line_per_generate(prompts, tmp_path):
    import json
    path = tmp_path / "m.jsonl"
    llm = _llm(metrics_path=str(path))
    sp = SamplingParams(temperature=0, max_tokens=4, ignore_eos=True)
    out = llm.generate(prompts[:2], sp)
    assert isinstance(out, list) and len(out) == 2  # return type unchanged without return_metrics
    res = llm.generate(prompts[:1], sp, return_metrics=True)
    rows = [json.loads(x) for x in path.read_text().splitlines()]
    assert [r["num_seqs"] for r in rows] == [2, 1] and [r["generated_tokens"] for r in rows] == [8, 4]
    assert rows[1]["throughput_tok_s"] == res["metrics"]["throughput_tok_s"] and "time" in rows[1]
