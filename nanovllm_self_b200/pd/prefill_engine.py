"""Prefill engine: runs prompts to their first token, then hands the sequence off.

Reference: ``pd_self/prefill_engine.py:9-265``.  Same behaviour: a sequence is handed off
when ``is_prefill_done and num_completion_tokens >= 1`` (:102-104); the payload carries
the prompt plus the first token and ``num_cached_tokens`` = the KV actually written;
``save_kv`` exports its KV; the sequence leaves ``running``, its session prefix is saved
and its prefill blocks are freed (:157-183).  A request whose ``max_tokens == 1``
finishes on the prefill side and yields ``finished=True`` with no transfer metadata.
"""
from __future__ import annotations

from ..engine.scheduler import Scheduler
from ..engine.sequence import Sequence, SequenceStatus
from ..sampling_params import SamplingParams
from .payload import HandoffPayload


class PrefillEngine:
    def __init__(self, config, tokenizer, model_runner, kv_connector):
        self.config = config
        self.tokenizer = tokenizer
        self.model_runner = model_runner
        self.kv_connector = kv_connector
        self.scheduler = Scheduler(config, model_runner.block_manager)
        self.last_step_scheduled = []

    # ---------------------------------------------------------------- inputs
    def _ids(self, text) -> list:
        if isinstance(text, str):
            if self.tokenizer is None:
                raise RuntimeError("text prompts need a tokenizer")
            return self.tokenizer(text, add_special_tokens=False)["input_ids"]
        return [int(t) for t in text]

    def _build_sequence(self, text, seq_idx, temperature, max_tokens, ignore_eos, session_id=None, top_p=1.0):
        sp = SamplingParams(temperature=temperature, max_tokens=max_tokens, ignore_eos=ignore_eos, top_p=top_p)
        return Sequence(seq_idx, self._ids(text), sp, self.config.block_size, session_id=session_id)

    def build_sequences(self, texts, temperature=0.0, max_tokens=64, ignore_eos=True, start_seq_id=0,
                        session_ids=None):
        return [self._build_sequence(t, start_seq_id + i, temperature, max_tokens, ignore_eos,
                                     session_ids[i] if session_ids is not None else None)
                for i, t in enumerate(texts)]

    def add_request(self, text, seq_idx: int, temperature: float = 0.0, max_tokens: int = 64,
                    ignore_eos: bool = True, request_id: str | None = None, session_id: str | None = None,
                    check_admission: bool = False) -> Sequence:
        seq = self._build_sequence(text, seq_idx, temperature, max_tokens, ignore_eos, session_id)
        seq.request_id = request_id or f"req-{seq_idx}"
        if check_admission and not self.scheduler.can_admit(seq):
            raise RuntimeError("server overloaded")
        self.scheduler.add(seq)
        return seq

    # --------------------------------------------------------------- handoff
    def _make_payload(self, seq: Sequence, finished: bool) -> HandoffPayload:
        meta = None if finished else self.kv_connector.save_kv(seq)
        return HandoffPayload(
            seq_idx=seq.seq_idx, request_id=seq.request_id or f"req-{seq.seq_idx}", token_ids=list(seq.token_ids),
            num_prompt_tokens=seq.num_prompt_tokens, num_cached_tokens=seq.num_cached_tokens,
            temperature=seq.temperature, max_tokens=seq.max_tokens, ignore_eos=seq.ignore_eos, finished=finished,
            transfer_meta=meta, session_id=seq.session_id, top_p=seq.top_p,
            prefix_cache_hit=bool(seq.prefix_cache_hit), prefix_cached_tokens=int(seq.prefix_cached_tokens),
            prefix_cache_source=seq.prefix_cache_source)

    @staticmethod
    def _is_handoff_ready(seq: Sequence) -> bool:
        return seq.is_prefill_done and seq.num_completion_tokens >= 1

    def step(self) -> list:
        seqs = self.scheduler.schedule()
        self.last_step_scheduled = seqs
        if not seqs:
            return []
        token_ids, need = self.model_runner.run(seqs)
        finished = self.scheduler.postprocess(seqs, token_ids, need)
        payloads = [self._make_payload(s, finished=True) for s in finished]
        for seq in list(self.scheduler.running):
            if seq.status != SequenceStatus.FINISHED and self._is_handoff_ready(seq):
                payloads.append(self._make_payload(seq, finished=False))
                self.scheduler.running.remove(seq)
                if seq.session_id:
                    self.model_runner.block_manager.save_session_prefix_cache(seq.session_id, seq)
                self.model_runner.block_manager.deallocate(seq)
                seq.status = SequenceStatus.FINISHED
        return payloads

    def run_prefill(self, texts, temperature=0.0, max_tokens=64, ignore_eos=True, start_seq_id=0,
                    max_empty_steps: int = 10000, session_ids=None) -> list:
        for i, t in enumerate(texts):
            self.add_request(t, start_seq_id + i, temperature, max_tokens, ignore_eos,
                             session_id=session_ids[i] if session_ids else None)
        out, empty = [], 0
        while not self.scheduler.is_finished():
            got = self.step()
            if not self.last_step_scheduled:
                empty += 1
                if empty > max_empty_steps:
                    raise RuntimeError(f"prefill made no progress: {self.scheduler.last_schedule_info.reason}")
                continue
            empty = 0
            out.extend(got)
        return sorted(out, key=lambda p: p.seq_idx)

    def abort_by_request_id(self, request_id: str) -> bool:
        for q in (self.scheduler.waiting, self.scheduler.running):
            for seq in list(q):
                if seq.request_id == request_id:
                    self.scheduler.abort(seq)
                    return True
        return False
