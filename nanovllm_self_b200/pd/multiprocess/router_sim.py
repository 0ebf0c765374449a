"""Routing-policy simulation: no GPU, no workers, only the router's service-time model.

Reference: ``pd_self/multiprocess/evaluation/benchmark_agent_load_scheduler.py`` (a pure-CPU comparison of
the routing policies on an agent trace).  Every request of a trace is routed by :class:`Router` at its
arrival time, all at t = 0 (``burst``) or one every 1 / rate seconds (``rate``).  The router's virtual
worker clocks then give each request its start, finish and queue wait under the model
``service = 0.02 + input / 4000 + output / 14 + ...`` (``agent_scheduler.service_time_s``).  Each policy
gets its own router over the same trace.  The summary per policy:
- makespan and generated tok/s;
- e2e and queue-wait percentiles;
- worker busy time and imbalance;
- affinity hit rate.

Each policy is also compared against ``round_robin``.

``python -m nanovllm_self_b200.pd.multiprocess.router_sim --workers 4 --trace agent --arrival burst``
"""
from __future__ import annotations

import argparse
import json

from .agent_scheduler import POLICIES, Router, RouterConfig, estimate


def quantile(xs: list, q: float) -> float:
    """Linear-interpolation quantile (q in [0, 1]) of a non-empty list."""
    s = sorted(xs)
    pos = q * (len(s) - 1)
    lo = int(pos)
    hi = min(lo + 1, len(s) - 1)
    return s[lo] + (s[hi] - s[lo]) * (pos - lo)


def _stats(xs: list) -> dict:
    return {"avg": sum(xs) / len(xs), "p50": quantile(xs, 0.5), "p90": quantile(xs, 0.9), "p99": quantile(xs, 0.99),
            "max": max(xs)}


def simulate(rows: list, num_workers: int, policy: str, arrival: str = "burst", rate: float = 4.0,
             cfg: RouterConfig | None = None, initial_backlog_s: list | None = None) -> dict:
    """Route every row of the trace with one policy; returns the per-request decisions and a summary."""
    if arrival not in ("burst", "rate"):
        raise ValueError(f"arrival must be 'burst' or 'rate', got {arrival!r}")
    if arrival == "rate" and rate <= 0:
        raise ValueError("rate must be positive")
    cfg = cfg or RouterConfig()
    router = Router(num_workers, policy, cfg, initial_backlog_s)
    decisions = []
    for i, row in enumerate(rows):
        now = 0.0 if arrival == "burst" else i / rate
        req = estimate(row, i, int(row["max_tokens"]), cfg)
        d = router.route(req, now)
        d.update(request_id=req.request_id, task_type=req.task_type, input_tokens=req.input_tokens,
                 output_tokens=req.output_tokens)
        decisions.append(d)
    if not decisions:
        return {"policy": policy, "decisions": [], "summary": {"num_requests": 0}}
    makespan = max(d["finish_time_s"] for d in decisions) - min(d["arrival_time_s"] for d in decisions)
    out_tokens = sum(d["output_tokens"] for d in decisions)
    sessions = {}
    for d in decisions:
        sessions.setdefault(d["session_id"], []).append(d)
    repeat = [d for ds in sessions.values() for d in ds[1:]]  # requests whose session was seen before
    summary = {"num_requests": len(decisions), "num_workers": num_workers, "arrival": arrival,
               "rate": rate if arrival == "rate" else None, "generated_tokens": out_tokens,
               "makespan_s": makespan, "generated_tok_s": out_tokens / makespan if makespan > 0 else 0.0,
               "e2e_s": _stats([d["estimated_e2e_time_s"] for d in decisions]),
               "queue_wait_s": _stats([d["queue_wait_time_s"] for d in decisions]),
               "service_s": _stats([d["estimated_service_time_s"] for d in decisions]),
               "affinity_hit_rate": (sum(1 for d in repeat if d["affinity_hit"]) / len(repeat)) if repeat else 0.0,
               **router.summary()}
    return {"policy": policy, "decisions": decisions, "summary": summary}


def compare(rows: list, num_workers: int, arrival: str = "burst", rate: float = 4.0,
            cfg: RouterConfig | None = None, policies=POLICIES) -> dict:
    """Every policy on the same trace, and each one's ratios against round_robin."""
    res = {p: simulate(rows, num_workers, p, arrival, rate, cfg)["summary"] for p in policies}
    base = res.get("round_robin")
    ratios = {}
    if base and base["num_requests"]:
        div = lambda a, b: a / b if b else None  # noqa: E731
        for p, s in res.items():
            if p == "round_robin":
                continue
            ratios[p] = {"tok_s_over_round_robin": div(s["generated_tok_s"], base["generated_tok_s"]),
                         "avg_e2e_over_round_robin": div(s["e2e_s"]["avg"], base["e2e_s"]["avg"]),
                         "p90_e2e_over_round_robin": div(s["e2e_s"]["p90"], base["e2e_s"]["p90"]),
                         "p99_e2e_over_round_robin": div(s["e2e_s"]["p99"], base["e2e_s"]["p99"]),
                         "avg_queue_over_round_robin": div(s["queue_wait_s"]["avg"], base["queue_wait_s"]["avg"])}
    return {"policies": res, "vs_round_robin": ratios}


def _trace(name: str, n: int, seed: int) -> list:
    from ...benchmarks import datasets
    if name == "agent":
        sessions = max(1, n // 4)
        return datasets.agent_sessions(sessions, vocab=1000, prefix_len=512, turns=4, seed=seed)[:n]
    if name == "lognormal":
        return datasets.pd_lognormal(n, vocab=1000, seed=seed)
    if name == "uniform":
        return datasets.uniform_serving(n, 1000, seed=seed)
    raise ValueError(f"unknown trace {name!r}")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--workers", type=int, default=4)
    ap.add_argument("--trace", choices=("agent", "lognormal", "uniform"), default="agent")
    ap.add_argument("--requests", type=int, default=200)
    ap.add_argument("--arrival", choices=("burst", "rate"), default="burst")
    ap.add_argument("--rate", type=float, default=4.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--prefill-tokens-per-s", type=float, default=RouterConfig.prefill_tokens_per_s)
    ap.add_argument("--decode-tokens-per-s", type=float, default=RouterConfig.decode_tokens_per_s)
    ap.add_argument("--affinity-max-extra-wait-s", type=float, default=RouterConfig.affinity_max_extra_wait_s)
    a = ap.parse_args(argv)
    cfg = RouterConfig(prefill_tokens_per_s=a.prefill_tokens_per_s, decode_tokens_per_s=a.decode_tokens_per_s,
                       affinity_max_extra_wait_s=a.affinity_max_extra_wait_s)
    rows = _trace(a.trace, a.requests, a.seed)
    out = compare(rows, a.workers, a.arrival, a.rate, cfg)
    out.update(bench="router_sim", trace=a.trace, requests=len(rows))
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
