"""Stage-1 regressions on the tiny random-init model (CPU, fp32), against the dense no-cache
oracle: the reference's ``tests/test_stage1_regression.py:149-191`` (prefill top-k equal to the
oracle's, greedy tokens unchanged when the KV block size changes, prompts one token either side
of a block boundary) with the oracle standing in for HuggingFace."""
import pytest
import torch

from nanovllm_self_b200 import LLM, SamplingParams
from nanovllm_self_b200.models.reference import dense_logits, greedy_generate

SP = dict(temperature=0, ignore_eos=True)


def _llm(block_size=16, **kw):
    base = dict(device="cpu", dtype="fp32", block_size=block_size, max_model_len=512,
                num_blocks=2 * 512 // block_size + 8)
    base.update(kw)
    return LLM("tiny", **base)


def _prompt(n, seed=11):
    return torch.randint(0, 1024, (n,), generator=torch.Generator().manual_seed(seed)).tolist()


@pytest.mark.parametrize("n", [7, 40])
def test_prefill_topk_matches_oracle(n):
    llm = _llm()
    p = _prompt(n)
    llm.add_request(p, SamplingParams(max_tokens=1, **SP))
    seqs = llm.scheduler.schedule()
    got = llm.model_runner.logits(seqs)[-1]
    want = dense_logits(llm.model_runner.model, p)
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-4)
    g, w = got.topk(10).indices.tolist(), want.topk(10).indices.tolist()
    assert g[0] == w[0] and set(g) == set(w)


def test_block_size_does_not_change_greedy_tokens():
    prompts = [_prompt(23, 1), _prompt(50, 2)]
    outs = []
    for bs in (4, 16, 256):
        llm = _llm(bs)
        outs.append([o[len(p):] for o, p in zip(llm.generate(prompts, SamplingParams(max_tokens=64, **SP)), prompts)])
    assert outs[0] == outs[1] == outs[2]
    model = _llm().model_runner.model
    assert outs[1] == [greedy_generate(model, p, 64) for p in prompts]


def test_prompts_at_block_boundaries_match_oracle():
    llm = _llm(16)
    prompts = [_prompt(n, 100 + n) for n in (15, 16, 17, 31, 32, 33)]
    out = llm.generate(prompts, SamplingParams(max_tokens=16, **SP))
    model = llm.model_runner.model
    for p, o in zip(prompts, out):
        assert o[len(p):] == greedy_generate(model, p, 16), len(p)
