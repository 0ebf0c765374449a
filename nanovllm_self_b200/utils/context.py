"""Per-step attention/batch metadata, passed explicitly (no global).

Fields follow the reference ``Context`` (``nanovllm/utils/context.py:4-36``):
``cu_seqlens_q``, ``cu_seqlens_k``, ``max_seqlen_q``, ``max_seqlen_k``,
``slot_mapping``, ``context_lens``, ``block_tables``, ``seq_need_compute_logits``.

Additions used by the B200 kernels:

* ``num_decode_seqs``: the batch is ordered decode-first (one query token each), so
  sequences ``[0, num_decode_seqs)`` take the split-KV decode kernel and the rest take
  the prefix-aware prefill kernel;
* ``logits_indices``: token row of the last token of each sampling sequence
  (``cu_seqlens_q[i + 1] - 1``), computed on the host;
* ``positions`` is carried by the runner, not here.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class Context:
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None
    seq_need_compute_logits: torch.Tensor | None = None
    logits_indices: torch.Tensor | None = None
    num_decode_seqs: int = 0
    num_seqs: int = 0
    num_tokens: int = 0
    # Host copies (optional) used by the CPU reference attention.
    host_q_lens: list | None = None
    host_k_lens: list | None = None
    kv_scales: tuple | None = None


def get_context(cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0, slot_mapping=None,
                context_lens=None, block_tables=None, seq_need_compute_logits=None, **kw) -> Context:
    return Context(cu_seqlens_q=cu_seqlens_q, cu_seqlens_k=cu_seqlens_k, max_seqlen_q=max_seqlen_q,
                   max_seqlen_k=max_seqlen_k, slot_mapping=slot_mapping, context_lens=context_lens,
                   block_tables=block_tables, seq_need_compute_logits=seq_need_compute_logits, **kw)
