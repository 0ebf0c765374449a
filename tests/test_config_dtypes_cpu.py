"""dtype aliases and the KV-cache dtype matrix on CPU (the reference's
``pd_self/evaluation/test_kv_cache_dtype_matrix.py:35-108``): aliases resolve, the runner allocates
the KV pool in the configured dtype, stores cast into it, and offline and online P/D run on it and
agree."""
import pytest
import torch

from nanovllm_self_b200 import LLM, SamplingParams
from nanovllm_self_b200.config import EngineConfig, resolve_torch_dtype
from nanovllm_self_b200.pd.coordinator import PDCoordinator
from nanovllm_self_b200.pd.online_coordinator import OnlinePDCoordinator


@pytest.mark.parametrize("alias,want", [("bf16", torch.bfloat16), ("bfloat16", torch.bfloat16),
                                        ("fp16", torch.float16), ("float16", torch.float16),
                                        ("fp32", torch.float32), ("float32", torch.float32),
                                        (torch.float16, torch.float16), ("auto", None), (None, None)])
def test_alias_resolution(alias, want):
    assert resolve_torch_dtype(alias) == want


def test_bad_alias_and_modes_are_rejected():
    with pytest.raises(ValueError):
        resolve_torch_dtype("fp13")
    with pytest.raises(ValueError):
        EngineConfig(kv_cache_quant_mode="int4")
    with pytest.raises(ValueError):
        EngineConfig(block_size=24)


def _cfg(**kw):
    base = dict(model="tiny", device="cpu", dtype="fp32", block_size=16, max_model_len=256, num_blocks=32)
    base.update(kw)
    return EngineConfig(**base)


@pytest.mark.parametrize("kw,kv_dtype,scales", [
    ({}, torch.float32, False),
    ({"kv_cache_dtype": "fp16"}, torch.float16, False),
    ({"kv_cache_dtype": "bf16"}, torch.bfloat16, False),
    ({"kv_cache_quant_mode": "int8_mock"}, torch.int8, True),
    ({"kv_cache_quant_mode": "fp8"}, torch.float8_e4m3fn, True),
])
def test_runner_binds_the_kv_dtype_and_stores_cast(kw, kv_dtype, scales):
    cfg = _cfg(**kw)
    assert cfg.kv_cache_dtype == kv_dtype
    llm = LLM(config=cfg)
    mr = llm.model_runner
    assert mr.kv_cache.dtype == kv_dtype and (mr.kv_scale_cache is not None) == scales
    prompt = torch.randint(0, 1024, (21,), generator=torch.Generator().manual_seed(2)).tolist()
    out = llm.generate([prompt], SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True))[0]
    assert len(out) == len(prompt) + 5
    assert mr.kv_cache.float().abs().sum() > 0  # the prompt's keys and values were stored in kv_dtype


@pytest.mark.parametrize("kv", ["fp16", "bf16"])
def test_online_pd_runs_on_a_reduced_precision_kv_cache(kv):
    prompts = [torch.randint(0, 1024, (n,), generator=torch.Generator().manual_seed(n)).tolist() for n in (9, 26)]
    want = PDCoordinator(_cfg(kv_cache_dtype=kv)).generate(prompts, max_tokens=6)
    oc = OnlinePDCoordinator(_cfg(kv_cache_dtype=kv))
    assert oc.decode_runner.kv_cache.dtype == resolve_torch_dtype(kv)
    assert oc.generate(prompts, max_tokens=6) == want
