"""Agent-aware request router for replicated P/D pairs or a P/D pool.

Reference: ``pd_self/multiprocess/agent_scheduler.py`` (policies ``round_robin``,
``load_aware`` and ``affinity_load_aware``).  The estimates follow the reference so the
policies rank workers the same way:

* task type from prompt keywords or length thresholds (tool_like / long_context /
  decode_heavy / simple_qa / mixed_agent);
* complexity = 0.3 * input + 1.0 * output + 64 * tool calls + 32 * extra steps;
* service time = 0.02 + input / 4000 + output / 14 + 0.3 * tools + 0.05 * extra steps (s);
* load-aware score = queue wait + projected finish + complexity / 10000, where queue wait
  adds the worker's real feedback load (``worker_state.json``) to its virtual clock;
* affinity: stay on the session's previous worker unless that costs more than 2 s of
  extra wait, otherwise move and re-pin.
"""
from __future__ import annotations

from dataclasses import dataclass, field

POLICIES = ("round_robin", "load_aware", "affinity_load_aware")
TOOL_WORDS = ("search", "calculate", "weather", "python", "code", "api", "database", "file")


@dataclass
class RouterConfig:
    short_input_threshold: int = 256
    long_input_threshold: int = 1024
    short_output_threshold: int = 128
    long_output_threshold: int = 128
    prefill_complexity_weight: float = 0.3
    decode_complexity_weight: float = 1.0
    tool_complexity_weight: float = 64.0
    step_complexity_weight: float = 32.0
    prefill_tokens_per_s: float = 4000.0
    decode_tokens_per_s: float = 14.0
    base_request_overhead_s: float = 0.02
    tool_call_time_s: float = 0.30
    step_overhead_s: float = 0.05
    queue_weight: float = 1.0
    finish_time_weight: float = 1.0
    complexity_capacity: float = 10000.0
    affinity_max_extra_wait_s: float = 2.0


# Reference names.
AgentSchedulerConfig = RouterConfig


@dataclass
class RequestEstimate:
    request_index: int
    request_id: str
    session_id: str
    task_type: str
    input_tokens: int
    output_tokens: int
    tool_calls: int
    steps: int
    complexity: float
    profile: str | None = None


@dataclass
class WorkerLoad:
    worker_id: int
    available_at_s: float = 0.0
    busy_time_s: float = 0.0
    num_requests: int = 0
    generated_tokens: int = 0
    feedback_load_s: float = 0.0
    feedback_state: dict | None = None

    def wait_s(self, now_s: float) -> float:
        return max(0.0, self.available_at_s - now_s) + self.feedback_load_s


def session_of(row: dict, request_id: str) -> str:
    for k in ("program_id", "session_id", "conversation_id", "source_id"):
        if row.get(k):
            return str(row[k])
    return request_id


def task_type_of(prompt, input_tokens: int, output_tokens: int, cfg: RouterConfig) -> str:
    text = str(prompt).lower()
    if any(w in text for w in TOOL_WORDS):
        return "tool_like"
    if input_tokens >= cfg.long_input_threshold:
        return "long_context"
    if output_tokens >= cfg.long_output_threshold:
        return "decode_heavy"
    if input_tokens <= cfg.short_input_threshold and output_tokens <= cfg.short_output_threshold:
        return "simple_qa"
    return "mixed_agent"


def estimate(row: dict, index: int, output_tokens: int, cfg: RouterConfig) -> RequestEstimate:
    n_in = int(row.get("input_tokens", len(row.get("prompt_ids", []) or [])))
    rid = row.get("id", f"agent-{index:06d}")
    ttype = row.get("task_type") or task_type_of(row.get("prompt", ""), n_in, output_tokens, cfg)
    tools = 1 if ttype == "tool_like" else 0
    steps = 1 + (n_in >= cfg.long_input_threshold) + (output_tokens >= cfg.long_output_threshold) + tools
    cx = (n_in * cfg.prefill_complexity_weight + output_tokens * cfg.decode_complexity_weight
          + tools * cfg.tool_complexity_weight + max(0, steps - 1) * cfg.step_complexity_weight)
    return RequestEstimate(index, rid, session_of(row, rid), ttype, n_in, output_tokens, tools, steps, cx,
                           row.get("profile"))


def service_time_s(req: RequestEstimate, cfg: RouterConfig) -> float:
    return (cfg.base_request_overhead_s + req.input_tokens / cfg.prefill_tokens_per_s
            + req.output_tokens / cfg.decode_tokens_per_s + req.tool_calls * cfg.tool_call_time_s
            + max(0, req.steps - 1) * cfg.step_overhead_s)


@dataclass
class Router:
    num_workers: int
    policy: str = "load_aware"
    cfg: RouterConfig = field(default_factory=RouterConfig)
    initial_backlog_s: list | None = None

    def __post_init__(self):
        if self.policy not in POLICIES:
            raise ValueError(f"unknown policy {self.policy!r}; choose from {POLICIES}")
        back = self.initial_backlog_s or [0.0] * self.num_workers
        if len(back) != self.num_workers:
            raise ValueError(f"expected {self.num_workers} initial backlogs, got {len(back)}")
        self.workers = [WorkerLoad(i, available_at_s=b, busy_time_s=b) for i, b in enumerate(back)]
        self.session_to_worker: dict[str, int] = {}

    def _score(self, w: WorkerLoad, req: RequestEstimate, now_s: float, svc: float) -> float:
        finish = max(w.available_at_s, now_s) + svc
        return (w.wait_s(now_s) * self.cfg.queue_weight + finish * self.cfg.finish_time_weight
                + req.complexity / self.cfg.complexity_capacity)

    def _best(self, req, now_s, svc) -> WorkerLoad:
        return min(self.workers, key=lambda w: (self._score(w, req, now_s, svc), w.worker_id))

    def update_feedback(self, worker_id: int, load_s: float, state: dict | None = None) -> None:
        self.workers[worker_id].feedback_load_s = float(load_s)
        self.workers[worker_id].feedback_state = state

    def route(self, req: RequestEstimate, now_s: float) -> dict:
        svc = service_time_s(req, self.cfg)
        hit, preferred = False, None
        if self.policy == "round_robin":
            w = self.workers[req.request_index % self.num_workers]
        elif self.policy == "load_aware":
            w = self._best(req, now_s, svc)
        else:
            best = self._best(req, now_s, svc)
            preferred = self.session_to_worker.get(req.session_id)
            if preferred is None:
                self.session_to_worker[req.session_id] = best.worker_id
                w = best
            else:
                pw = self.workers[preferred]
                if pw.wait_s(now_s) - best.wait_s(now_s) <= self.cfg.affinity_max_extra_wait_s:
                    w, hit = pw, True
                else:
                    self.session_to_worker[req.session_id] = best.worker_id
                    w = best
        start = max(now_s, w.available_at_s)
        finish = start + svc
        w.available_at_s = finish
        w.busy_time_s += svc
        w.num_requests += 1
        w.generated_tokens += req.output_tokens
        return {"worker_id": w.worker_id, "arrival_time_s": now_s, "start_time_s": start, "finish_time_s": finish,
                "queue_wait_time_s": start - now_s, "estimated_service_time_s": svc,
                "estimated_e2e_time_s": finish - now_s, "session_id": req.session_id, "affinity_hit": hit,
                "preferred_worker_id": preferred, "worker_feedback_load_s": w.feedback_load_s}

    def summary(self) -> dict:
        busy = [w.busy_time_s for w in self.workers]
        avg = sum(busy) / len(busy) if busy else 0.0
        return {"worker_busy_time_s": busy, "worker_num_requests": [w.num_requests for w in self.workers],
                "worker_generated_tokens": [w.generated_tokens for w in self.workers],
                "worker_feedback_load_s": [w.feedback_load_s for w in self.workers],
                "worker_load_imbalance": max(busy) / avg if avg > 0 else 0.0}
