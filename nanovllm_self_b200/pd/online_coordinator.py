"""Online P/D coordinator: request table, streaming token events, abort, per-step metrics.

Reference: ``pd_self/online_coordinator.py:12-376``.  ``submit`` admits a request (with
rollback on failure, duplicate ids rejected), ``step`` advances prefill by one step,
turns handoffs into first-token events, restores them into decode and advances decode by
one step; on an exception every active request is marked ERROR; ``stream(rid)`` yields
the events of one request; ``abort_request`` / ``finish_request`` clean up both sides.
"""
from __future__ import annotations

import uuid

from ..engine.sequence import SequenceStatus
from .coordinator import PDCoordinator
from .request_state import TERMINAL, RequestState, RequestStatus, TokenEvent
from .runtime_types import OnlineSchedulerStepMetrics


class OnlinePDCoordinator(PDCoordinator):
    def __init__(self, config, kv_backend: str = "dict", **kw):
        super().__init__(config, kv_backend, **kw)
        self.requests: dict[str, RequestState] = {}
        self.step_id = 0
        self.metrics_history: list[OnlineSchedulerStepMetrics] = []
        self._pending_payloads = []

    # ---------------------------------------------------------------- submit
    def submit(self, text, max_tokens: int = 64, temperature: float = 0.0, ignore_eos: bool = True,
               request_id: str | None = None, session_id: str | None = None, check_admission: bool = False) -> str:
        rid = request_id or uuid.uuid4().hex
        if rid in self.requests:
            raise ValueError(f"duplicate request_id {rid}")
        seq_idx = self._next_seq
        self._next_seq += 1
        ids = self.prefill_engine._ids(text)
        state = RequestState(rid, seq_idx, text, list(ids), temperature=temperature, max_tokens=max_tokens,
                             ignore_eos=ignore_eos, session_id=session_id)
        self.requests[rid] = state
        try:
            self.prefill_engine.add_request(ids, seq_idx, temperature, max_tokens, ignore_eos, request_id=rid,
                                            session_id=session_id, check_admission=check_admission)
        except Exception:
            self.requests.pop(rid, None)
            raise
        state.status = RequestStatus.PREFILLING
        return rid

    # ------------------------------------------------------------------ step
    def step(self) -> list:
        events = []
        try:
            payloads = self.prefill_engine.step()
            for p in payloads:
                st = self.requests.get(p.request_id)
                if st is None or st.is_terminal:
                    self.consumer.discard(p.transfer_meta)
                    continue
                events.append(st.emit(p.token_ids[-1]))
                if p.finished:
                    st.mark_finished("length" if len(st.output_ids) >= st.max_tokens else "stop")
                    continue
                st.handoff_payload = p
                st.status = RequestStatus.WAITING_DECODE
                self._pending_payloads.append(p)
            while self._pending_payloads:
                p = self._pending_payloads[0]
                st = self.requests[p.request_id]
                if not self.decode_runner.block_manager.num_free_blocks() >= (
                        p.transfer_meta.num_kv_blocks if p.transfer_meta else 0) + 1:
                    break
                self._pending_payloads.pop(0)
                self.decode_engine.restore_active_payload(p)
                st.status = RequestStatus.DECODING
            out = self.decode_engine.continuous_step()
            events.extend(self._collect_decode_events(out))
        except Exception as e:  # fail every live request loudly; the coordinator stays usable
            self._mark_active_requests_error(e)
            raise
        finally:
            self.step_id += 1
            self.record_online_scheduler_metrics(len(events))
        return events

    def _collect_decode_events(self, decode_out) -> list:
        events = []
        for i, tok in zip(decode_out.seq_need_compute_logits, decode_out.token_ids):
            seq = decode_out.scheduled[i]
            st = self.requests.get(seq.request_id)
            if st is None or st.is_terminal:
                continue
            events.append(st.emit(tok))
            if seq.status == SequenceStatus.FINISHED:
                st.mark_finished(seq.finish_reason or "length")
        return events

    # --------------------------------------------------------------- queries
    def is_finished(self, request_id: str) -> bool:
        st = self.requests.get(request_id)
        return st is None or st.is_terminal

    def has_unfinished(self) -> bool:
        return any(not s.is_terminal for s in self.requests.values())

    def stream(self, request_id: str, max_steps: int = 1_000_000):
        st = self.requests[request_id]
        steps = 0
        while True:
            while not st.stream_queue.empty():
                ev = st.stream_queue.get()
                yield ev
                if ev.finished:
                    return
            if steps >= max_steps:
                raise RuntimeError("stream made no progress")
            self.step()
            steps += 1

    def poll_events(self, request_id: str) -> list:
        st = self.requests[request_id]
        out = []
        while not st.stream_queue.empty():
            out.append(st.stream_queue.get())
        return out

    def count_requests_by_status(self) -> dict:
        counts = {s: 0 for s in RequestStatus}
        for st in self.requests.values():
            counts[st.status] += 1
        return counts

    def record_online_scheduler_metrics(self, emitted_events: int) -> None:
        pi = self.prefill_engine.scheduler.last_schedule_info
        di = self.decode_engine.scheduler.last_schedule_info
        c = self.count_requests_by_status()
        pu = self.prefill_runner.block_manager.get_block_usage_snapshot()
        du = self.decode_runner.block_manager.get_block_usage_snapshot()
        self.metrics_history.append(OnlineSchedulerStepMetrics(
            step_id=self.step_id, emitted_events=emitted_events,
            prefill_scheduled_decode_tokens=pi.num_decode_tokens, prefill_scheduled_prefill_tokens=pi.num_prefill_tokens,
            prefill_schedule_reason=pi.reason, decode_scheduled_decode_tokens=di.num_decode_tokens,
            decode_scheduled_prefill_tokens=di.num_prefill_tokens, decode_schedule_reason=di.reason,
            waiting_prefill_requests=len(self.prefill_engine.scheduler.waiting),
            prefill_running_sequences=len(self.prefill_engine.scheduler.running),
            decode_running_sequences=len(self.decode_engine.scheduler.running),
            finished_requests=c[RequestStatus.FINISHED], aborted_requests=c[RequestStatus.ABORTED],
            error_requests=c[RequestStatus.ERROR], prefill_used_blocks=pu["used_blocks"],
            prefill_free_blocks=pu["free_blocks"], decode_used_blocks=du["used_blocks"],
            decode_free_blocks=du["free_blocks"]))

    def get_last_online_scheduler_metrics(self):
        return self.metrics_history[-1] if self.metrics_history else None

    # ------------------------------------------------------------- lifecycle
    def _cleanup_request_resources(self, state: RequestState) -> None:
        self.prefill_engine.abort_by_request_id(state.request_id)
        self.decode_engine.abort_by_request_id(state.request_id)
        for p in list(self._pending_payloads):
            if p.request_id == state.request_id:
                self._pending_payloads.remove(p)
                self._cleanup_payload(p)

    def _cleanup_payload(self, payload) -> None:
        if payload is not None and payload.transfer_meta is not None:
            self.consumer.discard(payload.transfer_meta)

    def abort_request(self, request_id: str, reason: str = "abort") -> bool:
        st = self.requests.get(request_id)
        if st is None or st.is_terminal:
            return False
        self._cleanup_request_resources(st)
        st.mark_aborted(reason)
        return True

    def finish_request(self, request_id: str, finish_reason: str = "stop") -> None:
        st = self.requests.get(request_id)
        if st is None or st.is_terminal:
            return
        self._cleanup_request_resources(st)
        st.mark_finished(finish_reason)

    def _mark_active_requests_error(self, error) -> None:
        for st in self.requests.values():
            if not st.is_terminal:
                self._cleanup_request_resources(st)
                st.mark_error(error)

    def generate(self, texts, max_tokens=64, temperature=0.0, ignore_eos=True, max_steps: int = 100000):
        rids = [self.submit(t, max_tokens, temperature, ignore_eos) for t in texts]
        steps = 0
        while any(not self.is_finished(r) for r in rids):
            self.step()
            steps += 1
            if steps > max_steps:
                raise RuntimeError("online generate made no progress")
        return [self.requests[r].token_ids for r in rids]

    def request_metrics(self) -> dict:
        import numpy as np
        ttft = [s.ttft_s * 1e3 for s in self.requests.values() if s.ttft_s is not None]
        tpot = [s.tpot_s * 1e3 for s in self.requests.values() if s.tpot_s is not None]
        pct = lambda xs, q: float(np.percentile(xs, q)) if xs else 0.0  # noqa: E731
        return {"ttft_ms_p50": pct(ttft, 50), "ttft_ms_p99": pct(ttft, 99), "tpot_ms_p50": pct(tpot, 50),
                "tpot_ms_p99": pct(tpot, 99), "num_requests": len(self.requests)}
