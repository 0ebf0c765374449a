"""Decode engine: restores handed-off sequences into its own KV pool and decodes them.

Reference: ``pd_self/decode_engine.py:53-546``.  ``restore_sequence`` rebuilds the
``Sequence`` from the payload, allocates ``num_kv_blocks`` local blocks, loads the KV
through the connector and re-registers the full blocks' hash chain so later requests can
hit them (:232-275, :415-448); on failure it frees the blocks and discards the handoff.
``step`` / ``run_decode`` decode in batches; the continuous mode
(``restore_active_payload`` + ``continuous_step``) tracks per-request timings.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

from ..engine.scheduler import Scheduler
from ..engine.sequence import Sequence, SequenceStatus
from ..sampling_params import SamplingParams
from .runtime_types import DecodeStepOutput


@dataclass
class ActiveDecodeRequest:
    request_id: str
    seq: Sequence
    restore_time_s: float = 0.0
    start_time: float = field(default_factory=time.perf_counter)
    step_wall_s: list = field(default_factory=list)
    step_amortized_s: list = field(default_factory=list)
    payload_path: str | None = None

    @property
    def decode_time_s(self) -> float:
        return sum(self.step_wall_s)


class DecodeEngine:
    def __init__(self, config, tokenizer, model_runner, kv_connector):
        self.config = config
        self.tokenizer = tokenizer
        self.model_runner = model_runner
        self.kv_connector = kv_connector
        self.scheduler = Scheduler(config, model_runner.block_manager)
        self.active: dict[str, ActiveDecodeRequest] = {}
        self.finished_active: list[ActiveDecodeRequest] = []

    # --------------------------------------------------------------- restore
    def _allocate_local_blocks(self, payload) -> list:
        n = payload.transfer_meta.num_kv_blocks if payload.transfer_meta is not None else 0
        return self.model_runner.block_manager.allocate_block(n) if n else []

    def _restore_block_manager_meta(self, seq: Sequence) -> None:
        self.model_runner.block_manager.register_full_blocks(seq, seq.num_cached_tokens)

    def _new_sequence(self, payload) -> Sequence:
        sp = SamplingParams(temperature=payload.temperature, max_tokens=payload.max_tokens,
                            ignore_eos=payload.ignore_eos, top_p=getattr(payload, "top_p", 1.0))
        seq = Sequence(payload.seq_idx, payload.token_ids, sp, self.config.block_size,
                       session_id=getattr(payload, "session_id", None))
        seq.request_id = payload.request_id
        seq.num_prompt_tokens = payload.num_prompt_tokens
        seq.num_prefill_tokens = payload.num_cached_tokens
        seq.num_cached_tokens = payload.num_cached_tokens
        seq.status = SequenceStatus.RUNNING
        seq.first_token_time = time.perf_counter()
        return seq

    def restore_sequence(self, payload) -> Sequence:
        seq = self._new_sequence(payload)
        blocks = self._allocate_local_blocks(payload)
        seq.block_table = blocks
        try:
            if payload.transfer_meta is not None:
                self.kv_connector.load_kv(payload.transfer_meta, blocks)
            self._restore_block_manager_meta(seq)
        except Exception:
            self.model_runner.block_manager.free_blocks(blocks)
            seq.block_table = []
            self.kv_connector.discard(payload.transfer_meta)
            raise
        return seq

    def restore_sequence_from_kv_item(self, payload, kv_item) -> Sequence:
        seq = self._new_sequence(payload)
        blocks = self._allocate_local_blocks(payload)
        seq.block_table = blocks
        try:
            self.kv_connector.load_kv_item(kv_item, blocks)
            self._restore_block_manager_meta(seq)
        except Exception:
            self.model_runner.block_manager.free_blocks(blocks)
            seq.block_table = []
            raise
        return seq

    def restore_payloads(self, payloads) -> list:
        seqs = []
        for p in payloads:
            if p.finished:
                continue
            seq = self.restore_sequence(p)
            self.scheduler.running.append(seq)
            seqs.append(seq)
        return seqs

    def restore_active_payload(self, payload, payload_path: str | None = None) -> ActiveDecodeRequest:
        t0 = time.perf_counter()
        seq = self.restore_sequence(payload)
        self.scheduler.running.append(seq)
        req = ActiveDecodeRequest(payload.request_id, seq, time.perf_counter() - t0, payload_path=payload_path)
        self.active[payload.request_id] = req
        return req

    def restore_active_payload_from_kv_item(self, payload, kv_item, payload_path: str | None = None):
        t0 = time.perf_counter()
        seq = self.restore_sequence_from_kv_item(payload, kv_item)
        self.scheduler.running.append(seq)
        req = ActiveDecodeRequest(payload.request_id, seq, time.perf_counter() - t0, payload_path=payload_path)
        self.active[payload.request_id] = req
        return req

    # ------------------------------------------------------------------ step
    def step(self) -> DecodeStepOutput:
        seqs = self.scheduler.schedule()
        if not seqs:
            return DecodeStepOutput([], [], [], [])
        token_ids, need = self.model_runner.run(seqs)
        finished = self.scheduler.postprocess(seqs, token_ids, need)
        return DecodeStepOutput(seqs, token_ids, need, [s.seq_idx for s in finished])

    def continuous_step(self) -> DecodeStepOutput:
        t0 = time.perf_counter()
        out = self.step()
        wall = time.perf_counter() - t0
        if out.scheduled:
            share = wall / len(out.scheduled)
            for s in out.scheduled:
                req = self.active.get(s.request_id)
                if req is not None:
                    req.step_wall_s.append(wall)
                    req.step_amortized_s.append(share)
        for s in out.scheduled:
            if s.status == SequenceStatus.FINISHED and s.request_id in self.active:
                self.finished_active.append(self.active.pop(s.request_id))
        return out

    def run_decode(self, payloads, max_empty_steps: int = 10000) -> dict:
        seqs = self.restore_payloads(payloads)
        empty = 0
        while not self.scheduler.is_finished():
            out = self.step()
            if not out.scheduled:
                empty += 1
                if empty > max_empty_steps:
                    raise RuntimeError(f"decode made no progress: {self.scheduler.last_schedule_info.reason}")
                continue
            empty = 0
        results = {s.request_id: list(s.token_ids) for s in seqs}
        for p in payloads:
            if p.finished:
                results[p.request_id] = list(p.token_ids)
        return results

    def cleanup_sequence(self, seq: Sequence) -> None:
        self.scheduler.abort(seq)

    def abort_by_request_id(self, request_id: str) -> bool:
        for q in (self.scheduler.waiting, self.scheduler.running):
            for seq in list(q):
                if seq.request_id == request_id:
                    self.scheduler.abort(seq)
                    self.active.pop(request_id, None)
                    return True
        return False
