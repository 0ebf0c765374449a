"""LLM backends for the agent: ``generate_text(prompt, max_tokens, metadata) -> str``.

Reference: ``claude_self/backend.py`` (local engine), ``scheduled_backend.py`` (router in
front of several engines), ``pd_pool_backend.py`` (the multiprocess P/D pool) and the
test-only ``FakeBackend``.
"""
from __future__ import annotations

import time

from ..sampling_params import SamplingParams


class ByteTokenizer:
    """Fallback text codec for checkpoints without a tokenizer: one id per UTF-8 byte."""
    eos_token_id = None

    def encode(self, text: str) -> list:
        return list(text.encode("utf-8"))

    def decode(self, ids) -> str:
        return bytes(int(i) % 256 for i in ids).decode("utf-8", errors="replace")


def _codec(llm):
    tok = getattr(llm, "tokenizer", None)
    if tok is not None:
        return (lambda t: tok(t, add_special_tokens=False)["input_ids"]), \
               (lambda ids: tok.decode(ids, skip_special_tokens=True))
    b = ByteTokenizer()
    return b.encode, b.decode


class LocalBackend:
    """One in-process engine; the agent's session id turns on the session prefix cache."""

    def __init__(self, llm, temperature: float = 0.0):
        self.llm = llm
        self.temperature = temperature
        self.encode, self.decode = _codec(llm)

    def generate_text(self, prompt: str, max_tokens: int = 256, metadata: dict | None = None) -> str:
        ids = self.encode(prompt)
        out = self.llm.generate([ids], SamplingParams(temperature=self.temperature, max_tokens=max_tokens),
                                request_metadata=metadata)[0]
        return self.decode(out[len(ids):])


class ScheduledBackend:
    """Routes each call to one of several engines with the agent-aware router."""

    def __init__(self, engines: list, policy: str = "affinity_load_aware", temperature: float = 0.0):
        from ..pd.multiprocess.agent_scheduler import Router
        self.backends = [LocalBackend(e, temperature) for e in engines]
        self.router = Router(len(engines), policy)
        self.calls = 0
        self.t0 = time.time()
        self.routes = []

    def generate_text(self, prompt: str, max_tokens: int = 256, metadata: dict | None = None) -> str:
        from ..pd.multiprocess.agent_scheduler import RouterConfig, estimate
        meta = dict(metadata or {})
        row = {"id": f"agent-{self.calls}", "prompt": prompt, "input_tokens": len(self.backends[0].encode(prompt)),
               "session_id": meta.get("session_id"), "task_type": meta.get("task_type")}
        est = estimate(row, self.calls, max_tokens, RouterConfig())
        route = self.router.route(est, time.time() - self.t0)
        self.routes.append(route)
        self.calls += 1
        return self.backends[route["worker_id"]].generate_text(prompt, max_tokens, meta)


class PDPoolBackend:
    """Sends each call through a running :class:`~nanovllm_self_b200.pd.multiprocess.pool.PDPool`."""

    def __init__(self, pool, encode=None, decode=None, timeout_s: float = 600.0):
        b = ByteTokenizer()
        self.pool = pool
        self.encode = encode or b.encode
        self.decode = decode or b.decode
        self.timeout_s = timeout_s
        self.calls = 0
        self.t0 = time.time()

    def generate_text(self, prompt: str, max_tokens: int = 256, metadata: dict | None = None) -> str:
        meta = metadata or {}
        ids = self.encode(prompt)
        row = {"id": f"agent-{self.calls}", "prompt": prompt, "prompt_ids": ids, "max_tokens": max_tokens,
               "input_tokens": len(ids), "session_id": meta.get("session_id"), "task_type": meta.get("task_type")}
        base = self.pool.submit(row, self.calls, time.time() - self.t0)
        self.calls += 1
        deadline = time.time() + self.timeout_s
        while base not in self.pool.results:
            self.pool._collect()
            if time.time() > deadline:
                raise TimeoutError("P/D pool did not answer")
            time.sleep(0.002)
        res = self.pool.results[base]
        if "error" in res:
            raise RuntimeError(res["error"])
        return self.decode(res["output_ids"])


class FakeBackend:
    """Scripted backend for tests: returns the given replies in order and records every call."""

    def __init__(self, replies: list):
        self.replies = list(replies)
        self.calls = []

    def generate_text(self, prompt: str, max_tokens: int = 128, metadata: dict | None = None) -> str:
        self.calls.append({"prompt": prompt, "max_tokens": max_tokens, "metadata": dict(metadata or {})})
        return self.replies[min(len(self.calls) - 1, len(self.replies) - 1)]
