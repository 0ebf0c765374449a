"""Service-side request lifecycle (reference ``pd_self/request_state.py``).

``RequestState`` is the serving object (status, output ids, a stream queue of
``TokenEvent``); ``Sequence`` stays the execution object.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum, auto
from queue import Queue
from time import perf_counter
from typing import Optional

from .payload import HandoffPayload


class RequestStatus(Enum):
    WAITING_PREFILL = auto()
    PREFILLING = auto()
    WAITING_DECODE = auto()
    DECODING = auto()
    FINISHED = auto()
    ABORTED = auto()
    ERROR = auto()


TERMINAL = (RequestStatus.FINISHED, RequestStatus.ABORTED, RequestStatus.ERROR)


@dataclass
class TokenEvent:
    request_id: str
    token_id: int | None
    text: str = ""
    finished: bool = False
    finish_reason: str | None = None
    error: str | None = None


@dataclass
class RequestState:
    request_id: str
    seq_idx: int
    prompt: object
    input_ids: list
    output_ids: list = field(default_factory=list)
    temperature: float = 0.0
    max_tokens: int = 64
    ignore_eos: bool = True
    session_id: Optional[str] = None
    status: RequestStatus = RequestStatus.WAITING_PREFILL
    handoff_payload: Optional[HandoffPayload] = None
    stream_queue: Queue = field(default_factory=Queue)
    created_time: float = field(default_factory=perf_counter)
    first_token_time: float | None = None
    token_times: list = field(default_factory=list)
    finished_time: float | None = None
    error: str | None = None

    @property
    def token_ids(self) -> list:
        return self.input_ids + self.output_ids

    @property
    def is_terminal(self) -> bool:
        return self.status in TERMINAL

    def emit(self, token_id: int) -> TokenEvent:
        now = perf_counter()
        if self.first_token_time is None:
            self.first_token_time = now
        self.token_times.append(now)
        self.output_ids.append(int(token_id))
        ev = TokenEvent(self.request_id, int(token_id))
        self.stream_queue.put(ev)
        return ev

    def mark_finished(self, finish_reason: str = "stop"):
        self.status = RequestStatus.FINISHED
        self.finished_time = perf_counter()
        self.stream_queue.put(TokenEvent(self.request_id, None, finished=True, finish_reason=finish_reason))

    def mark_aborted(self, reason: str = "abort"):
        self.status = RequestStatus.ABORTED
        self.finished_time = perf_counter()
        self.stream_queue.put(TokenEvent(self.request_id, None, finished=True, finish_reason=reason))

    def mark_error(self, error):
        self.status = RequestStatus.ERROR
        self.error = str(error)
        self.finished_time = perf_counter()
        self.stream_queue.put(TokenEvent(self.request_id, None, finished=True, finish_reason="error",
                                         error=str(error)))

    @property
    def ttft_s(self) -> float | None:
        return None if self.first_token_time is None else self.first_token_time - self.created_time

    @property
    def tpot_s(self) -> float | None:
        if len(self.token_times) < 2:
            return None
        return (self.token_times[-1] - self.token_times[0]) / (len(self.token_times) - 1)
