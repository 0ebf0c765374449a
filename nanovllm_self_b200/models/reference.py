"""Dense, no-KV-cache Qwen3 forward: the correctness oracle.

Replaces the reference's HuggingFace ``generate`` oracle
(``tests/test_compare_with_hf.py:39-44``): with random weights and no checkpoint the
oracle is a from-scratch full-sequence forward of the same weights, recomputing the
whole prefix for every generated token.  Works at TP=1 on any device.
"""
from __future__ import annotations

import torch

from ..ops import torch_ref as R
from .qwen3 import Qwen3ForCausalLM


@torch.inference_mode()
def dense_logits(model: Qwen3ForCausalLM, token_ids: list[int]) -> torch.Tensor:
    """Logits [V] of the last position for one sequence (fp32)."""
    assert model.tp_size == 1
    dev = model.device
    ids = torch.as_tensor(token_ids, dtype=torch.long, device=dev)
    pos = torch.arange(len(token_ids), device=dev)
    nq, nkv, d = model.num_heads, model.num_kv_heads, model.head_dim
    x = R.embedding(ids, model.embed)
    for L in model.layers:
        h = R.rmsnorm(x, L.ln1, model.eps)
        qkv = R.linear(h, L.qkv)
        q = qkv[:, :nq * d].reshape(-1, nq, d)
        k = qkv[:, nq * d:(nq + nkv) * d].reshape(-1, nkv, d)
        v = qkv[:, (nq + nkv) * d:].reshape(-1, nkv, d)
        q = R.apply_rope(R.rmsnorm(q, L.q_norm, model.eps), pos, model.cos_sin)
        k = R.apply_rope(R.rmsnorm(k, L.k_norm, model.eps), pos, model.cos_sin)
        o = R.dense_causal_attention(q, k, v, model.scale).reshape(-1, nq * d)
        x = (x.float() + R.linear(o, L.o).float()).to(x.dtype)
        h = R.rmsnorm(x, L.ln2, model.eps)
        a = R.silu_mul_interleaved(R.linear(h, L.gate_up)).to(x.dtype)
        x = (x.float() + R.linear(a, L.down).float()).to(x.dtype)
    x = R.rmsnorm(x[-1:], model.norm, model.eps)
    return R.linear(x, model.lm_head)[0].float()


@torch.inference_mode()
def greedy_generate(model: Qwen3ForCausalLM, prompt: list[int], max_tokens: int) -> list[int]:
    toks = list(prompt)
    for _ in range(max_tokens):
        toks.append(int(dense_logits(model, toks).argmax()))
    return toks[len(prompt):]
