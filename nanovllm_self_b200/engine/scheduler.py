"""Token-budget scheduler: decode first, then running prefill chunks, then admission.

Behaviour follows the reference ``Scheduler`` (``nanovllm/engine/scheduler.py:23-283``):

1. every running sequence whose prefill is done gets one decode token
   (``can_append`` then ``may_append``);
2. running sequences still in prefill advance by their remaining prompt, capped by
   ``prefill_chunk_size`` when chunked prefill is on and by the token budget;
3. waiting sequences are admitted FIFO (``can_allocate`` then ``allocate``); admission
   stops at the first sequence that does not fit.

``postprocess`` appends the sampled token only to sequences that sampled this step,
finishes on ``eos`` (unless ``ignore_eos``) or ``max_tokens``, saves the session prefix
before freeing, and then advances ``num_cached_tokens`` for all others.

Added on top of the reference (which never preempts and so stalls when the KV pool is
exhausted, reference :211-218): when a decode cannot get a block, the newest running
sequence is preempted (its blocks freed, recomputed later from the front of the
waiting queue).  ``enable_preemption=False`` restores the reference's behaviour.
"""
from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field

from .block_manager import BlockManager
from .sequence import Sequence, SequenceStatus


@dataclass
class ScheduleOutput:
    seqs: list = field(default_factory=list)
    decode_seqs: list = field(default_factory=list)
    prefill_seqs: list = field(default_factory=list)
    new_prefill_seqs: list = field(default_factory=list)
    num_decode_tokens: int = 0
    num_prefill_tokens: int = 0
    token_budget_used: int = 0
    token_budget_remaining: int = 0
    blocked_decode: int = 0
    blocked_prefill: int = 0
    num_preempted: int = 0
    reason: str = "ok"


class Scheduler:
    def __init__(self, config, block_manager: BlockManager):
        self.config = config
        self.block_manager = block_manager
        self.max_num_seqs = config.max_num_seqs
        self.max_num_batched_tokens = config.max_num_batched_tokens
        self.eos = config.eos
        self.enable_preemption = getattr(config, "enable_preemption", True)
        self.waiting: deque[Sequence] = deque()
        self.running: deque[Sequence] = deque()
        self.num_preemptions = 0
        self.last_schedule_info = ScheduleOutput(token_budget_remaining=self.max_num_batched_tokens,
                                                 reason="idle")

    def add(self, seq: Sequence) -> None:
        self.waiting.append(seq)

    def can_admit(self, seq: Sequence) -> bool:
        return self.block_manager.can_allocate(seq)

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def num_unfinished(self) -> int:
        return len(self.waiting) + len(self.running)

    # ---------------------------------------------------------------- schedule
    def _chunk(self, seq: Sequence, budget: int) -> int:
        n = seq.num_prefill_tokens - seq.num_cached_tokens
        if self.config.enable_chunked_prefill:
            n = min(n, self.config.prefill_chunk_size)
        return min(n, budget)

    def _preempt(self, seq: Sequence) -> None:
        self.block_manager.deallocate(seq)
        seq.status = SequenceStatus.WAITING
        seq.num_new_tokens = 0
        seq.num_cached_tokens = 0
        seq.num_prefill_tokens = len(seq.token_ids)
        seq.num_preemptions += 1
        self.num_preemptions += 1
        if seq in self.running:
            self.running.remove(seq)
        self.waiting.appendleft(seq)

    # Reference name (never called by the reference itself).
    preempty = _preempt

    def schedule(self) -> list[Sequence]:
        bm = self.block_manager
        decode, prefill, new = [], [], []
        blocked_decode = blocked_prefill = preempted = 0
        num_seqs = 0
        budget = self.max_num_batched_tokens
        initial = budget

        # 1. decode first
        for seq in list(self.running):
            if budget <= 0 or num_seqs >= self.max_num_seqs:
                break
            if seq.status == SequenceStatus.WAITING or not seq.is_prefill_done:
                continue
            while not bm.can_append(seq):
                victim = None
                if self.enable_preemption:
                    for cand in reversed(self.running):
                        if cand is not seq and cand not in decode:
                            victim = cand
                            break
                if victim is None:
                    break
                self._preempt(victim)
                preempted += 1
            if not bm.can_append(seq):
                if self.enable_preemption and not decode:
                    # Nothing else to evict: recompute this one later.
                    self._preempt(seq)
                    preempted += 1
                else:
                    blocked_decode += 1
                    seq.blocked_reason = "no_free_block_for_decode"
                continue
            bm.may_append(seq)
            seq.num_new_tokens = 1
            seq.status = SequenceStatus.RUNNING
            seq.blocked_reason = None
            decode.append(seq)
            budget -= 1
            num_seqs += 1

        # 2. running prefills (chunks)
        for seq in list(self.running):
            if budget <= 0 or num_seqs >= self.max_num_seqs:
                break
            if seq.is_prefill_done:
                continue
            n = self._chunk(seq, budget)
            if n <= 0:
                continue
            seq.num_new_tokens = n
            seq.status = SequenceStatus.RUNNING
            seq.blocked_reason = None
            prefill.append(seq)
            budget -= n
            num_seqs += 1

        # 3. admit waiting FIFO (no admission while decodes are starved of blocks)
        while self.waiting and budget > 0 and num_seqs < self.max_num_seqs and not blocked_decode:
            seq = self.waiting[0]
            if not seq.block_table:
                if not bm.can_allocate(seq):
                    blocked_prefill += 1
                    seq.blocked_reason = "no_free_block_for_prefill"
                    break
                bm.allocate(seq)
            n = self._chunk(seq, budget)
            if n <= 0:
                break
            seq.num_new_tokens = n
            seq.status = SequenceStatus.RUNNING
            seq.blocked_reason = None
            self.waiting.popleft()
            self.running.append(seq)
            new.append(seq)
            budget -= n
            num_seqs += 1

        scheduled = decode + prefill + new
        reason = "ok"
        if not scheduled:
            if blocked_decode or blocked_prefill:
                reason = "blocked_by_blocks"
            elif budget <= 0:
                reason = "token_budget_exhausted"
            elif num_seqs >= self.max_num_seqs:
                reason = "seq_budget_exhausted"
            elif self.waiting or self.running:
                reason = "no_runnable_seq"
            else:
                reason = "idle"
        self.last_schedule_info = ScheduleOutput(
            seqs=scheduled, decode_seqs=decode, prefill_seqs=prefill, new_prefill_seqs=new,
            num_decode_tokens=len(decode),
            num_prefill_tokens=sum(s.num_new_tokens for s in prefill) + sum(s.num_new_tokens for s in new),
            token_budget_used=initial - budget, token_budget_remaining=budget,
            blocked_decode=blocked_decode, blocked_prefill=blocked_prefill,
            num_preempted=preempted, reason=reason)
        return scheduled

    # ------------------------------------------------------------ postprocess
    def postprocess(self, seqs: list[Sequence], token_ids: list[int], seq_need_compute_logits: list[int]):
        assert len(token_ids) == len(seq_need_compute_logits)
        finished = []
        now = time.perf_counter()
        for idx, tok in zip(seq_need_compute_logits, token_ids):
            seq = seqs[idx]
            seq.append_token(tok)
            if seq.first_token_time is None:
                seq.first_token_time = now
            if seq.token_times is not None:
                seq.token_times.append(now)
            hit_eos = (not seq.ignore_eos) and tok == self.eos
            if hit_eos or seq.num_completion_tokens >= seq.max_tokens:
                seq.status = SequenceStatus.FINISHED
                seq.finish_time = now
                seq.finish_reason = "stop" if hit_eos else "length"
                if seq.session_id:
                    self.block_manager.save_session_prefix_cache(seq.session_id, seq)
                self.block_manager.deallocate(seq)
                if seq in self.running:
                    self.running.remove(seq)
                finished.append(seq)
        for seq in seqs:
            if seq.status != SequenceStatus.FINISHED:
                seq.num_cached_tokens += seq.num_new_tokens
                seq.num_new_tokens = 0
        return finished

    # ------------------------------------------------------------------ abort
    def abort(self, seq: Sequence) -> None:
        if seq in self.waiting:
            self.waiting.remove(seq)
        if seq in self.running:
            self.running.remove(seq)
        self.block_manager.deallocate(seq)
        seq.status = SequenceStatus.FINISHED
        seq.finish_reason = "abort"
        seq.num_new_tokens = 0
        seq.blocked_reason = None

    def abort_by_seq_idx(self, seq_idx: int) -> bool:
        for q in (self.waiting, self.running):
            for seq in list(q):
                if seq.seq_idx == seq_idx:
                    self.abort(seq)
                    return True
        return False
