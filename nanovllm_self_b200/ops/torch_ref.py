"""Plain-PyTorch implementations of every hot op.

These run the tiny CPU model (fp32) and are the numerics oracle for the CUDA kernels
(each GPU kernel test compares against these evaluated in fp32).  They mirror the
reference's eager semantics:

* RMSNorm in fp32, cast back (``nanovllm/layers/RMSNorm.py:11-17``);
* NeoX rotate-half RoPE in fp32 with a ``[max_pos, D]`` cos‖sin table
  (``nanovllm/layers/RoPE.py:5-55``);
* KV store by slot ``block * BS + offset`` (``nanovllm/layers/attention.py:139-189``),
  with the cache laid out ``[num_blocks, kv_heads, block_size, head_dim]`` per layer;
* causal attention whose mask is offset by ``k_len - q_len`` so that a chunk or a
  prefix-hit prefill sees all cached tokens (``attention.py:378-498``);
* sampler: greedy for temperature <= 0, else softmax(logits / T) sampling, with an
  optional top-p filter (``nanovllm/layers/sampler.py:9-43``).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

FP8_MAX = 448.0
FP8_HEADROOM = 4.0


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * r * w.float()).to(x.dtype)


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor | None, w: torch.Tensor, eps: float):
    """residual' = x + residual (or x); returns (rmsnorm(residual'), residual')."""
    r = x if residual is None else (x.float() + residual.float()).to(x.dtype)
    return rmsnorm(r, w, eps), r


def rope_cos_sin(head_dim: int, max_pos: int, theta: float, device=None) -> torch.Tensor:
    """fp32 table [max_pos, head_dim]: first half cos, second half sin."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    return torch.cat([f.cos(), f.sin()], dim=-1).float().to(device)


def apply_rope(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """x [T, H, D] rotated by the NeoX rule at ``positions`` [T]."""
    d2 = x.shape[-1] // 2
    cs = cos_sin[positions.long()]
    cos, sin = cs[:, None, :d2], cs[:, None, d2:]
    x1, x2 = x.float()[..., :d2], x.float()[..., d2:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


def fp8_block_scale(first_token_absmax: torch.Tensor) -> torch.Tensor:
    return torch.clamp(first_token_absmax.float() * FP8_HEADROOM / FP8_MAX, min=1e-8)


def store_kv(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
             slot_mapping: torch.Tensor, k_scale: torch.Tensor | None = None,
             v_scale: torch.Tensor | None = None) -> None:
    """Scatter k, v [T, Hkv, D] into caches [NB, Hkv, BS, D] at ``slot_mapping`` [T].

    Negative slots are skipped (padding rows).  For fp8 caches the per-(block, head)
    scale is set by the step that writes the block's first token: absmax of that token
    times a headroom of 4, divided by 448; later tokens in the block reuse it.
    """
    bs = k_cache.shape[2]
    slots = slot_mapping.long()
    keep = slots >= 0
    if not bool(keep.all()):
        k, v, slots = k[keep], v[keep], slots[keep]
    blk, off = slots // bs, slots % bs
    if k_cache.dtype == torch.float8_e4m3fn:
        for cache, x, sc in ((k_cache, k, k_scale), (v_cache, v, v_scale)):
            first = off == 0
            if bool(first.any()):
                amax = x[first].float().abs().amax(dim=-1)  # [n_first, Hkv]
                sc[blk[first]] = fp8_block_scale(amax)
            s = sc[blk]  # [T, Hkv]
            q = torch.clamp(x.float() / s[..., None], -FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
            cache[blk, :, off] = q
    elif k_cache.dtype == torch.int8:
        for cache, x, sc in ((k_cache, k, k_scale), (v_cache, v, v_scale)):
            amax = x.float().abs().amax(dim=-1)
            s = torch.clamp(amax / 127.0, min=1e-6)
            qv = torch.clamp(torch.round(x.float() / s[..., None]), -127, 127).to(torch.int8)
            cache[blk, :, off] = qv
            sc[blk, :, off] = s
    else:
        k_cache[blk, :, off] = k.to(k_cache.dtype)
        v_cache[blk, :, off] = v.to(v_cache.dtype)


def gather_kv(cache: torch.Tensor, block_table, k_len: int, scale: torch.Tensor | None = None) -> torch.Tensor:
    """Return [k_len, Hkv, D] fp32 for one sequence."""
    bs = cache.shape[2]
    nb = (k_len + bs - 1) // bs
    ids = torch.as_tensor(list(block_table[:nb]), dtype=torch.long, device=cache.device)
    x = cache[ids].float()  # [nb, Hkv, BS, D]
    if cache.dtype == torch.float8_e4m3fn:
        x = x * scale[ids][:, :, None, None].float()
    elif cache.dtype == torch.int8:
        x = x * scale[ids][..., None].float()
    return x.permute(0, 2, 1, 3).reshape(nb * bs, x.shape[1], x.shape[3])[:k_len]


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    q_lens: list, k_lens: list, block_tables: list, scale: float,
                    k_scale=None, v_scale=None) -> torch.Tensor:
    """q [T, Hq, D] (sequences packed in order) -> out [T, Hq, D]."""
    out = torch.empty_like(q)
    hq, hkv = q.shape[1], k_cache.shape[1]
    g = hq // hkv
    t0 = 0
    for i, (ql, kl) in enumerate(zip(q_lens, k_lens)):
        if ql == 0:
            continue
        qi = q[t0:t0 + ql].float()  # [ql, Hq, D]
        k = gather_kv(k_cache, block_tables[i], kl, k_scale).repeat_interleave(g, dim=1)
        v = gather_kv(v_cache, block_tables[i], kl, v_scale).repeat_interleave(g, dim=1)
        s = torch.einsum("qhd,khd->hqk", qi, k) * scale
        qpos = torch.arange(ql, device=q.device)[:, None] + (kl - ql)
        kpos = torch.arange(kl, device=q.device)[None, :]
        s = s.masked_fill((kpos > qpos)[None], float("-inf"))
        p = torch.softmax(s, dim=-1)
        out[t0:t0 + ql] = torch.einsum("hqk,khd->qhd", p, v).to(q.dtype)
        t0 += ql
    return out


def silu_mul(x: torch.Tensor) -> torch.Tensor:
    """x [T, 2I] = gate ‖ up -> silu(gate) * up [T, I]."""
    i = x.shape[-1] // 2
    g, u = x[..., :i].float(), x[..., i:].float()
    return (F.silu(g) * u).to(x.dtype)


GATE_UP_GROUP = 16


def interleave_gate_up(g: torch.Tensor, u: torch.Tensor, group: int = GATE_UP_GROUP) -> torch.Tensor:
    """[I, H] gate and up weights -> [2I, H] with rows interleaved in groups of ``group``:
    rows 2·group·j .. +group-1 are gate features group·j.., the next ``group`` rows the
    matching up features.  Every tile of 32 output columns of ``x @ W^T`` then holds 16
    gates and their 16 ups, which lets the GEMM apply SiLU-and-mul in its epilogue."""
    i, h = g.shape
    if i % group:
        raise ValueError(f"intermediate size {i} is not a multiple of {group}")
    return torch.stack([g.reshape(i // group, group, h), u.reshape(i // group, group, h)], 1).reshape(2 * i, h)


def silu_mul_interleaved(y: torch.Tensor, group: int = GATE_UP_GROUP) -> torch.Tensor:
    """y [T, 2I] in the interleaved layout of :func:`interleave_gate_up` -> silu(gate) * up [T, I]."""
    t, n = y.shape
    y = y.float().reshape(t, n // (2 * group), 2, group)
    return (F.silu(y[:, :, 0]) * y[:, :, 1]).reshape(t, n // 2)


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return F.linear(x, w)


def embedding(ids: torch.Tensor, w: torch.Tensor, vocab_start: int = 0) -> torch.Tensor:
    """Rows of the (possibly vocab-sharded) table; ids outside the shard give zeros."""
    local = ids.long() - vocab_start
    ok = (local >= 0) & (local < w.shape[0])
    out = w[torch.where(ok, local, torch.zeros_like(local))]
    return out * ok[:, None].to(out.dtype)


def sample(logits: torch.Tensor, temperatures: torch.Tensor, top_p: torch.Tensor | None = None,
           generator: torch.Generator | None = None, batch_greedy_compat: bool = False) -> torch.Tensor:
    """Per-row: argmax if T <= 0 else sample softmax(logits / T) restricted to top-p."""
    logits = logits.float()
    greedy = logits.argmax(dim=-1)
    t = temperatures.float()
    if batch_greedy_compat and bool((t <= 0).any()):
        return greedy
    if bool((t <= 0).all()):
        return greedy
    probs = torch.softmax(logits / torch.where(t > 0, t, torch.ones_like(t))[:, None], dim=-1)
    if top_p is not None and bool((top_p < 1.0).any()):
        sp, si = probs.sort(dim=-1, descending=True)
        cum = sp.cumsum(-1)
        drop = (cum - sp) > top_p[:, None].float()
        sp = sp.masked_fill(drop, 0.0)
        probs = torch.zeros_like(probs).scatter_(-1, si, sp)
    drawn = torch.multinomial(probs, 1, generator=generator).squeeze(-1)
    return torch.where(t > 0, drawn, greedy)


def dense_causal_attention(q, k, v, scale):
    """No-cache attention for one sequence: q [L, Hq, D], k/v [L, Hkv, D]."""
    g = q.shape[1] // k.shape[1]
    k = k.repeat_interleave(g, dim=1).float()
    v = v.repeat_interleave(g, dim=1).float()
    s = torch.einsum("qhd,khd->hqk", q.float(), k) * scale
    L = q.shape[0]
    mask = torch.triu(torch.ones(L, L, dtype=torch.bool, device=q.device), 1)
    s = s.masked_fill(mask[None], float("-inf"))
    return torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).to(q.dtype)


def softmax_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
