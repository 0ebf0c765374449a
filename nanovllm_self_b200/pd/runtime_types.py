"""Step output / metrics records of the P/D engines (reference ``pd_self/runtime_types.py``)."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class DecodeStepOutput:
    scheduled: list
    token_ids: list
    seq_need_compute_logits: list
    finished_seq_ids: list


@dataclass
class OnlineSchedulerStepMetrics:
    step_id: int
    emitted_events: int
    prefill_scheduled_decode_tokens: int
    prefill_scheduled_prefill_tokens: int
    prefill_schedule_reason: str
    decode_scheduled_decode_tokens: int
    decode_scheduled_prefill_tokens: int
    decode_schedule_reason: str
    waiting_prefill_requests: int
    prefill_running_sequences: int
    decode_running_sequences: int
    finished_requests: int
    aborted_requests: int
    error_requests: int
    prefill_used_blocks: int
    prefill_free_blocks: int
    decode_used_blocks: int
    decode_free_blocks: int
