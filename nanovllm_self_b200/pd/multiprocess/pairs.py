"""Fixed P/D pairs routed by the agent-aware router, and the synthetic P/D pipeline benchmark.

Reference: ``pd_self/multiprocess/evaluation/benchmark_agent_pd_multi_pair.py:70-123`` (N
independent prefill/decode pairs, each its own worker pair and work directory, one router
choosing the PAIR per request from the request's estimate, the pairs' virtual backlogs and
their workers' live state files; closed-loop or batch submission; per-request metrics
rows and a summary), ``compare_agent_pd_pool_strategies.py`` (the routing policies side by
side on the same requests) and ``benchmark_synthetic_pd_pipeline.py`` (one pair, synthetic
length-profile requests, warm-up requests, per-request metrics and percentiles).

Here a pair is a one-prefill, one-decode :class:`~.pool.PDPool` (any KV backend, any TP
size per worker) and :class:`PDPairs` routes over them; unlike the pool, a request's prefill
and decode stay in one pair, so the KV handoff never crosses pairs.  Run from the shell::

    python -m nanovllm_self_b200.pd.multiprocess.pairs --work-root /tmp/pairs --pairs 2 \
        --policies round_robin,load_aware,affinity_load_aware --num-requests 64

(``--pairs 1`` with the synthetic length profile is the pipeline benchmark).
"""
from __future__ import annotations

import argparse
import json
import time
from pathlib import Path

import numpy as np

from .agent_scheduler import POLICIES, Router, RouterConfig, estimate
from .pool import PDPool, _pct


class PDPairs:
    def __init__(self, work_root, num_pairs: int = 2, backend: str = "shared_memory", model: str = "tiny",
                 devices=None, policy: str = "affinity_load_aware", worker_args=None,
                 handshake_timeout_s: float = 120.0, nccl_port: int = 29800, tp: int = 1, device_kind: str = "cuda"):
        """``devices``: one (prefill device, decode device) per pair (default: GPUs 2i and 2i + 1,
        or with ``tp`` > 1 every worker a TP group of consecutive GPUs)."""
        self.root = Path(work_root)
        self.n = num_pairs
        self.pools = []
        for i in range(num_pairs):
            if tp > 1:
                # pair i: prefill group on GPUs [2 i tp, (2 i + 1) tp), decode group on the next tp
                kw = dict(tp=tp, device_kind=device_kind, gpu_base=2 * i * tp)
            else:
                pd = devices[i] if devices else (f"cuda:{2 * i}", f"cuda:{2 * i + 1}")
                kw = dict(prefill_devices=[pd[0]], decode_devices=[pd[1]])
            self.pools.append(PDPool(self.root / f"pair_{i}", 1, 1, backend, model, worker_args=worker_args,
                                     handshake_timeout_s=handshake_timeout_s, nccl_port=nccl_port + 10 * i, **kw))
        self.router = Router(num_pairs, policy)
        self.policy = policy
        self.submitted = {}  # key -> (pair, base, row, route)
        self.rows_out = []   # per-request metrics rows of the current run
        self._k = 0

    def start(self, ready_timeout_s: float = 600.0) -> None:
        for p in self.pools:
            p.start(ready_timeout_s)

    def shutdown(self) -> None:
        for p in self.pools:
            p.shutdown()

    def set_policy(self, policy: str) -> None:
        """A fresh router with `policy` (the workers keep running)."""
        self.router = Router(self.n, policy)
        self.policy = policy

    def _feedback(self) -> None:
        for i, p in enumerate(self.pools):
            load, state = 0.0, {}
            for role, wd in (("prefill", p.pwd[0]), ("decode", p.dwd[0])):
                try:
                    st = wd.read_json("worker_state.json")
                except (FileNotFoundError, json.JSONDecodeError):
                    continue
                state[role] = st
                load += st.get("queue_depth", 0) * 0.05 + st.get("active", 0) * 0.01 + st.get("pending_push", 0) * 0.01
                load += 0.02 if st.get("busy") else 0.0
            self.router.update_feedback(i, load, state)

    def submit(self, row: dict, index: int, now_s: float) -> str:
        self._feedback()
        est = estimate(row, index, int(row["max_tokens"]), RouterConfig())
        route = self.router.route(est, now_s)
        pair = route["worker_id"]
        base = self.pools[pair].submit(row, index, now_s)
        key = f"p{pair}:{base}"
        self.submitted[key] = (pair, base, row, dict(route, task_type=est.task_type))
        return key

    def _done(self, key: str) -> dict | None:
        pair, base, row, route = self.submitted[key]
        res = self.pools[pair].results.get(base)
        if res is None:
            return None
        out = {"request_id": row.get("id", key), "pair": pair, "policy": self.policy,
               "session_id": route.get("session_id"), "affinity_hit": bool(route.get("affinity_hit")),
               "task_type": route.get("task_type"), "input_tokens": len(row["prompt_ids"]),
               "max_tokens": row["max_tokens"]}
        if "error" in res:
            out["error"] = res["error"]
        else:
            out.update(output_tokens=len(res["output_ids"]), ttft_s=res["ttft_s"], tpot_s=res["tpot_s"],
                       e2e_s=res["e2e_s"], output_ids=res["output_ids"])
        return out

    def run(self, rows: list, concurrency: int | None = 4, rate: float | None = None, warmup: int = 0,
            timeout_s: float = 3600.0, request_timeout_s: float | None = None, seed: int = 0) -> dict:
        """Submit `rows` (closed loop at `concurrency`, or Poisson at `rate` req/s) after
        `warmup` unmeasured requests; returns the summary (metrics rows in ``rows_out``)."""
        import random
        if warmup:
            self._drive(rows[:warmup], concurrency or 1, None, timeout_s, request_timeout_s, random.Random(seed))
        self.rows_out = []
        t0 = time.time()
        self._drive(rows[warmup:], concurrency, rate, timeout_s, request_timeout_s, random.Random(seed + 1))
        wall = time.time() - t0
        ok = [r for r in self.rows_out if "error" not in r]
        gen = sum(r["output_tokens"] for r in ok)
        per_pair = [sum(1 for r in self.rows_out if r["pair"] == i) for i in range(self.n)]
        return {"policy": self.policy, "pairs": self.n, "num_requests": len(self.rows_out),
                "num_errors": len(self.rows_out) - len(ok), "wall_s": wall,
                "output_tok_s": gen / wall if wall > 0 else 0.0,
                "ttft_ms_p50": _pct([r["ttft_s"] * 1e3 for r in ok], 50),
                "ttft_ms_p99": _pct([r["ttft_s"] * 1e3 for r in ok], 99),
                "tpot_ms_p50": _pct([r["tpot_s"] * 1e3 for r in ok], 50),
                "tpot_ms_p99": _pct([r["tpot_s"] * 1e3 for r in ok], 99),
                "e2e_s_p90": _pct([r["e2e_s"] for r in ok], 90),
                "affinity_hit_rate": (sum(r["affinity_hit"] for r in self.rows_out) / len(self.rows_out)
                                      if self.rows_out else 0.0),
                "requests_per_pair": per_pair, "router": self.router.summary()}

    def _drive(self, rows, concurrency, rate, timeout_s, request_timeout_s, rng) -> None:
        t0 = time.time()
        next_arrival = 0.0
        i = 0
        inflight = set()
        while i < len(rows) or inflight:
            now = time.time() - t0
            if i < len(rows):
                if rate:
                    if now >= next_arrival:
                        inflight.add(self.submit(rows[i], self._k, now))
                        self._k += 1
                        i += 1
                        next_arrival += rng.expovariate(rate)
                elif len(inflight) < (concurrency or 1):
                    inflight.add(self.submit(rows[i], self._k, now))
                    self._k += 1
                    i += 1
            for p in self.pools:
                p._collect()
                live = {self.submitted[k][1] for k in inflight if self.submitted[k][0] == self.pools.index(p)}
                p._fail_stuck(live, request_timeout_s)
            for key in list(inflight):
                out = self._done(key)
                if out is not None:
                    inflight.discard(key)
                    self.rows_out.append(out)
            if time.time() - t0 > timeout_s:
                raise TimeoutError("P/D pairs run timed out")
            time.sleep(0.001)


def compare_policies(pairs: PDPairs, rows: list, policies=POLICIES, **run_kw) -> list:
    """The same requests under each routing policy, one summary per policy (same workers)."""
    out = []
    for pol in policies:
        pairs.set_policy(pol)
        out.append(pairs.run(rows, **run_kw))
    return out


def synthetic_rows(n: int, input_mean: float = 2048, output_mean: float = 256, sessions: int = 8, seed: int = 0,
                   vocab: int = 151936, sigma: float = 0.5, max_input: int = 8192, max_output: int = 1024) -> list:
    """Lognormal input / output lengths (clipped), random token ids, `sessions` round-robin sessions."""
    rng = np.random.default_rng(seed)
    rows = []
    for i in range(n):
        n_in = int(np.clip(rng.lognormal(np.log(input_mean), sigma), 16, max_input))
        n_out = int(np.clip(rng.lognormal(np.log(output_mean), sigma), 2, max_output))
        rows.append({"id": f"req-{i}", "prompt_ids": rng.integers(0, vocab, n_in).tolist(), "max_tokens": n_out,
                     "input_tokens": n_in, "session_id": f"s{i % sessions}"})
    return rows


def load_rows(path, limit: int | None = None) -> list:
    """Rows from a JSON-lines workload file (``benchmarks.datasets``), the first `limit` of them;
    every row gets an ``id`` and ``input_tokens`` if it has none."""
    rows = []
    with open(path) as f:
        for line in f:
            if not line.strip():
                continue
            r = json.loads(line)
            r.setdefault("id", f"req-{len(rows)}")
            r.setdefault("input_tokens", len(r["prompt_ids"]))
            rows.append(r)
            if limit is not None and len(rows) >= limit:
                break
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser(description="fixed P/D pairs / synthetic P/D pipeline benchmark")
    ap.add_argument("--work-root", required=True)
    ap.add_argument("--pairs", type=int, default=2)
    ap.add_argument("--backend", default="ipc_push")
    ap.add_argument("--model", default="qwen3-0.6b")
    ap.add_argument("--policies", default="affinity_load_aware")
    ap.add_argument("--num-requests", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--rate", type=float, default=None)
    ap.add_argument("--concurrency", type=int, default=4)
    ap.add_argument("--input-mean", type=float, default=2048)
    ap.add_argument("--output-mean", type=float, default=256)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--out", default=None, help="JSON summary path; per-request rows go to <out>.jsonl")
    ap.add_argument("--dataset", default=None, help="JSON-lines rows (benchmarks.datasets); default synthetic")
    args, rest = ap.parse_known_args(argv)
    if args.dataset:
        rows = load_rows(args.dataset, args.num_requests + args.warmup)
    else:
        rows = synthetic_rows(args.num_requests + args.warmup, args.input_mean, args.output_mean)
    pairs = PDPairs(args.work_root, args.pairs, args.backend, args.model, worker_args=rest, tp=args.tp)
    pairs.start()
    results, per_request = [], []
    try:
        for pol in args.policies.split(","):
            pairs.set_policy(pol)
            results.append(pairs.run(rows, concurrency=args.concurrency, rate=args.rate, warmup=args.warmup))
            per_request += pairs.rows_out
    finally:
        pairs.shutdown()
    for r in results:
        print(json.dumps(r))
    if args.out:
        with open(args.out, "w") as f:
            json.dump(results, f, indent=1)
        with open(args.out + ".jsonl", "w") as f:
            for r in per_request:
                f.write(json.dumps(r) + "\n")  # with output_ids: the correctness check compares them


if __name__ == "__main__":
    main()
