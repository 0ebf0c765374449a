"""Per-request execution state.

Behaviour follows the reference ``Sequence`` (``nanovllm/engine/Sequence.py:5-106``):

* ``num_cached_tokens`` is the progress pointer (tokens whose KV is in the cache),
  ``num_new_tokens`` is this step's advance, ``num_context_tokens = cached + new``;
* ``is_prefill_done`` once the whole prompt is cached;
* ``is_need_logits`` once this step reaches the end of ``token_ids`` (so a chunked
  prefill only samples on its last chunk).

Additions: ``arrival_time``/``first_token_time``/``finish_time`` for TTFT/TPOT, a
``num_preemptions`` counter, ``top_p`` and a per-request ``seed``.
"""
from __future__ import annotations

import time
from enum import Enum, auto

from ..sampling_params import SamplingParams


class SequenceStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()


class Sequence:
    __slots__ = (
        "seq_idx", "request_id", "session_id", "token_ids", "block_table", "block_size",
        "num_prompt_tokens", "num_cached_tokens", "num_new_tokens", "status",
        "blocked_reason", "temperature", "max_tokens", "ignore_eos", "top_p", "seed",
        "prefix_cache_hit", "prefix_cached_tokens", "prefix_new_tokens", "prefix_cache_source",
        "arrival_time", "first_token_time", "finish_time", "num_preemptions", "token_times",
        "finish_reason", "num_prefill_tokens",
    )

    def __init__(self, seq_idx: int, token_ids, sampling_params: SamplingParams | None = None,
                 block_size: int = 16, session_id: str | None = None):
        sp = sampling_params if sampling_params is not None else SamplingParams()
        self.seq_idx = seq_idx
        self.request_id = None
        self.session_id = session_id
        self.token_ids: list[int] = [int(t) for t in token_ids]
        if not self.token_ids:
            raise ValueError("a sequence needs at least one prompt token")
        self.block_table: list[int] = []
        self.block_size = block_size
        self.num_prompt_tokens = len(self.token_ids)
        # Tokens that must be in the KV cache before single-token decode starts: the
        # prompt, or every token so far after a preemption (recompute).
        self.num_prefill_tokens = self.num_prompt_tokens
        self.num_cached_tokens = 0
        self.num_new_tokens = 0
        self.status = SequenceStatus.WAITING
        self.blocked_reason = None
        self.temperature = float(sp.temperature)
        self.max_tokens = int(sp.max_tokens)
        self.ignore_eos = bool(sp.ignore_eos)
        self.top_p = float(getattr(sp, "top_p", 1.0))
        self.seed = getattr(sp, "seed", None)
        self.prefix_cache_hit = False
        self.prefix_cached_tokens = 0
        self.prefix_new_tokens = self.num_prompt_tokens
        self.prefix_cache_source = None
        self.arrival_time = time.perf_counter()
        self.first_token_time = None
        self.finish_time = None
        self.num_preemptions = 0
        self.token_times: list[float] | None = None
        self.finish_reason = None

    def __len__(self) -> int:
        return len(self.token_ids)

    def __getitem__(self, idx):
        return self.token_ids[idx]

    def __repr__(self) -> str:
        return (f"Sequence(idx={self.seq_idx}, len={len(self)}, cached={self.num_cached_tokens}, "
                f"new={self.num_new_tokens}, status={self.status.name})")

    @property
    def token_len(self) -> int:
        return len(self.token_ids)

    @property
    def last_token(self) -> int:
        return self.token_ids[-1]

    def append_token(self, token) -> None:
        self.token_ids.append(int(token))

    @property
    def num_prompt_remaining_tokens(self) -> int:
        return self.num_prefill_tokens - self.num_cached_tokens

    @property
    def is_prefill_done(self) -> bool:
        return self.num_cached_tokens >= self.num_prefill_tokens

    @property
    def num_context_tokens(self) -> int:
        return self.num_cached_tokens + self.num_new_tokens

    @property
    def num_blocks(self) -> int:
        return (len(self.token_ids) + self.block_size - 1) // self.block_size

    @property
    def last_block_num_tokens(self) -> int:
        rem = len(self.token_ids) % self.block_size
        return self.block_size if rem == 0 else rem

    @property
    def num_completion_tokens(self) -> int:
        return len(self.token_ids) - self.num_prompt_tokens

    @property
    def completion_token_ids(self) -> list[int]:
        return self.token_ids[self.num_prompt_tokens:]

    @property
    def is_need_logits(self) -> bool:
        return self.num_context_tokens == len(self.token_ids)

    @property
    def is_finished(self) -> bool:
        return self.status == SequenceStatus.FINISHED
