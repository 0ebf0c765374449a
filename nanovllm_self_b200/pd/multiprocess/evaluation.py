"""Single-engine baseline, single-vs-P/D comparison and per-request correctness check.

Reference counterparts, restated for this framework's per-request rows:

* ``pd_self/multiprocess/evaluation/benchmark_synthetic_single_gpu.py`` -- the synthetic
  requests served by one monolithic engine, the baseline a P/D run is compared with.
  Here :func:`run_single` drives :class:`~nanovllm_self_b200.engine.llm_engine.LLMEngine`
  through ``add_request`` / ``step`` with the same arrival process as the P/D drivers
  (closed loop at a concurrency, or Poisson at a rate), so both sides see the same load, and
  writes rows with the same fields as :class:`~.pairs.PDPairs` (``request_id``,
  ``input_tokens``, ``output_tokens``, ``ttft_s``, ``tpot_s``, ``e2e_s``, ``output_ids``).
* ``compare_synthetic_benchmark.py`` -- :func:`compare_summaries`: the P/D summary over the
  single-engine one (TTFT / TPOT percentiles, p90 end-to-end latency, throughput).
* ``compare_agent_pd_pool_strategies.py`` / ``compare_agent_pd_strategies.py`` --
  :func:`policy_report`: the routing policies' summaries (one :class:`~.pairs.PDPairs` or
  :class:`~.pool.PDPool` run per policy) side by side, each over ``round_robin``
  (throughput, TTFT, TPOT, p90 end-to-end), with affinity hits and the requests-per-pair
  imbalance, and :func:`markdown_table` for the report.
* ``check_pipeline_correctness.py:44-66`` -- :func:`check_correctness`: two runs' rows
  matched by request id; passed when both ran the same requests and every request's
  generated token ids are equal (times are never compared).  Used to check one KV backend,
  policy or pool shape against another, or a P/D run against the single engine.

Command line (rows are JSON lines, one per request; summaries are JSON)::

    python -m nanovllm_self_b200.pd.multiprocess.evaluation single --model qwen3-8b --out single.json
    python -m nanovllm_self_b200.pd.multiprocess.evaluation compare --single single.json --pd pd.json
    python -m nanovllm_self_b200.pd.multiprocess.evaluation correctness --left a.jsonl --right b.jsonl
    python -m nanovllm_self_b200.pd.multiprocess.evaluation policies --summaries pairs.json --markdown p.md
"""
from __future__ import annotations

import argparse
import json
import random
import time
from pathlib import Path

import torch

from .pool import _pct

RATIO_KEYS = ("ttft_ms_p50", "ttft_ms_p99", "tpot_ms_p50", "tpot_ms_p99", "e2e_s_p90", "output_tok_s", "wall_s")


def summarize(rows: list, wall_s: float, **extra) -> dict:
    """Summary of per-request rows in the P/D drivers' format (errors counted, not timed)."""
    ok = [r for r in rows if "error" not in r]
    gen = sum(r["output_tokens"] for r in ok)
    out = {"num_requests": len(rows), "num_errors": len(rows) - len(ok), "wall_s": wall_s,
           "output_tok_s": gen / wall_s if wall_s > 0 else 0.0,
           "ttft_ms_p50": _pct([r["ttft_s"] * 1e3 for r in ok], 50),
           "ttft_ms_p99": _pct([r["ttft_s"] * 1e3 for r in ok], 99),
           "tpot_ms_p50": _pct([r["tpot_s"] * 1e3 for r in ok], 50),
           "tpot_ms_p99": _pct([r["tpot_s"] * 1e3 for r in ok], 99),
           "e2e_s_p90": _pct([r["e2e_s"] for r in ok], 90)}
    out.update(extra)
    return out


def _drive(llm, rows: list, concurrency: int | None, rate: float | None, seed: int, timeout_s: float) -> list:
    """Serve `rows` on `llm`: admit at `rate` req/s (Poisson) or keep `concurrency` in flight;
    one engine step per loop turn.  Returns one row per request in completion order."""
    from ...sampling_params import SamplingParams
    rng = random.Random(seed)
    t0 = time.perf_counter()
    next_arrival, i = 0.0, 0
    inflight, out = {}, []
    with torch.inference_mode():
        while i < len(rows) or inflight:
            now = time.perf_counter() - t0
            while i < len(rows) and ((rate and now >= next_arrival) or
                                     (not rate and len(inflight) < (concurrency or 1))):
                r = rows[i]
                sp = SamplingParams(temperature=r.get("temperature", 0.0), max_tokens=int(r["max_tokens"]),
                                    ignore_eos=r.get("ignore_eos", True))
                seq = llm.add_request(r["prompt_ids"], sp, r.get("session_id"))
                inflight[seq.seq_idx] = (r, seq)
                i += 1
                if rate:
                    next_arrival += rng.expovariate(rate)
            if not inflight:
                time.sleep(min(0.001, max(0.0, next_arrival - now)))
                continue
            llm.step()
            for sid, (r, seq) in list(inflight.items()):
                if seq.finish_time is None:
                    continue
                del inflight[sid]
                n_out = seq.num_completion_tokens
                first = seq.first_token_time or seq.finish_time
                out.append({"request_id": r.get("id", f"req-{sid}"), "session_id": r.get("session_id"),
                            "input_tokens": len(r["prompt_ids"]), "max_tokens": r["max_tokens"],
                            "output_tokens": n_out, "ttft_s": first - seq.arrival_time,
                            "tpot_s": (seq.finish_time - first) / max(1, n_out - 1),
                            "e2e_s": seq.finish_time - seq.arrival_time,
                            "output_ids": list(seq.token_ids[seq.num_prompt_tokens:])})
            if time.perf_counter() - t0 > timeout_s:
                raise TimeoutError("single-engine run timed out")
    return out


def run_single(llm, rows: list, concurrency: int | None = 4, rate: float | None = None, warmup: int = 0,
               seed: int = 0, timeout_s: float = 3600.0) -> tuple[dict, list]:
    """The single-engine baseline: `warmup` unmeasured requests, then the rest under the same
    arrival process the P/D drivers use.  Returns (summary, per-request rows)."""
    if warmup:
        _drive(llm, rows[:warmup], concurrency or 1, None, seed, timeout_s)
    t0 = time.perf_counter()
    out = _drive(llm, rows[warmup:], concurrency, rate, seed + 1, timeout_s)
    return summarize(out, time.perf_counter() - t0, mode="single"), out


def compare_summaries(single: dict, pd: dict) -> dict:
    """P/D over single for every latency / throughput key both summaries have
    (``<key>_pd_over_single``; None where the single value is missing or zero)."""
    res = {"num_requests_single": single.get("num_requests"), "num_requests_pd": pd.get("num_requests"),
           "num_errors_single": single.get("num_errors"), "num_errors_pd": pd.get("num_errors")}
    for k in RATIO_KEYS:
        a, b = single.get(k), pd.get(k)
        if a is None or b is None:
            continue
        res[f"{k}_single"], res[f"{k}_pd"] = a, b
        res[f"{k}_pd_over_single"] = b / a if a else None
    return res


def policy_report(summaries: list, baseline: str = "round_robin") -> dict:
    """Each policy's summary next to the baseline policy's: latency and throughput, their ratios over
    the baseline (``*_over_<baseline>``), affinity hit rate and the requests-per-pair imbalance
    (largest pair over the mean; 1.0 is an even spread)."""
    base = next((x for x in summaries if x.get("policy") == baseline), summaries[0])
    bname = base.get("policy", baseline)
    rows = []
    for x in summaries:
        per = x.get("requests_per_pair") or []
        row = {"policy": x.get("policy"), "num_requests": x.get("num_requests"), "num_errors": x.get("num_errors")}
        for k in ("output_tok_s", "ttft_ms_p50", "ttft_ms_p99", "tpot_ms_p50", "tpot_ms_p99", "e2e_s_p90",
                  "affinity_hit_rate"):
            row[k] = x.get(k)
        row["requests_per_pair"] = per
        row["pair_imbalance"] = max(per) / (sum(per) / len(per)) if per and sum(per) else None
        for k in ("output_tok_s", "ttft_ms_p50", "tpot_ms_p50", "e2e_s_p90"):
            a, b = base.get(k), x.get(k)
            row[f"{k}_over_{bname}"] = b / a if a and b is not None else None
        rows.append(row)
    return {"baseline": bname, "policies": rows}


def markdown_table(report: dict) -> str:
    b = report["baseline"]
    head = ["policy", "tok/s", f"tok/s / {b}", "TTFT p50 ms", "TTFT p99 ms", "TPOT p50 ms", "e2e p90 s",
            "affinity hits", "pair imbalance", "errors"]

    def f(v, fmt="{:.2f}"):
        return "-" if v is None else fmt.format(v)
    lines = ["| " + " | ".join(head) + " |", "|" + "---|" * len(head)]
    for r in report["policies"]:
        lines.append("| " + " | ".join([str(r["policy"]), f(r["output_tok_s"], "{:.1f}"),
                                        f(r[f"output_tok_s_over_{b}"]), f(r["ttft_ms_p50"], "{:.1f}"),
                                        f(r["ttft_ms_p99"], "{:.1f}"), f(r["tpot_ms_p50"]), f(r["e2e_s_p90"]),
                                        f(r["affinity_hit_rate"]), f(r["pair_imbalance"]),
                                        str(r["num_errors"])]) + " |")
    return "\n".join(lines) + "\n"


def _by_id(rows: list) -> dict:
    return {r["request_id"]: r for r in rows if not r.get("warmup")}


def check_correctness(left: list, right: list, show: int = 20) -> dict:
    """Match two runs' rows by request id and compare generated token ids.  Passed when
    neither side misses a request the other has, neither side has an error row, and every
    common request generated the same tokens."""
    L, R = _by_id(left), _by_id(right)
    common = sorted(set(L) & set(R))
    mismatches, errors = [], []
    for rid in common:
        a, b = L[rid], R[rid]
        if "error" in a or "error" in b:
            errors.append({"request_id": rid, "left": a.get("error"), "right": b.get("error")})
            continue
        if a.get("output_ids") != b.get("output_ids"):
            x, y = a.get("output_ids") or [], b.get("output_ids") or []
            first = next((i for i, (u, v) in enumerate(zip(x, y)) if u != v), min(len(x), len(y)))
            mismatches.append({"request_id": rid, "first_divergence": first, "left_tokens": len(x),
                               "right_tokens": len(y)})
    miss_l, miss_r = sorted(set(R) - set(L)), sorted(set(L) - set(R))
    return {"num_left": len(L), "num_right": len(R), "num_common": len(common),
            "num_missing_left": len(miss_l), "num_missing_right": len(miss_r),
            "num_errors": len(errors), "num_mismatches": len(mismatches),
            "passed": not (miss_l or miss_r or errors or mismatches),
            "missing_left": miss_l[:show], "missing_right": miss_r[:show], "errors": errors[:show],
            "mismatches": mismatches[:show]}


def read_rows(path) -> list:
    with open(path) as f:
        return [json.loads(line) for line in f if line.strip()]


def write_rows(path, rows: list) -> None:
    with open(path, "w") as f:
        for r in rows:
            f.write(json.dumps(r) + "\n")


def main(argv=None):
    ap = argparse.ArgumentParser(description="single-engine baseline / single-vs-P/D comparison / correctness")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("single", help="serve the synthetic requests on one engine")
    s.add_argument("--model", default="qwen3-0.6b")
    s.add_argument("--device", default="cuda")
    s.add_argument("--dtype", default="bf16")
    s.add_argument("--num-requests", type=int, default=32)
    s.add_argument("--warmup", type=int, default=2)
    s.add_argument("--concurrency", type=int, default=4)
    s.add_argument("--rate", type=float, default=None)
    s.add_argument("--input-mean", type=float, default=2048)
    s.add_argument("--output-mean", type=float, default=256)
    s.add_argument("--max-model-len", type=int, default=9216)
    s.add_argument("--block-size", type=int, default=256)
    s.add_argument("--dataset", default=None, help="JSON-lines rows (benchmarks.datasets); default synthetic")
    s.add_argument("--out", default=None, help="summary JSON; rows go to <out>.jsonl")
    c = sub.add_parser("compare", help="P/D summary over the single-engine summary")
    c.add_argument("--single", required=True)
    c.add_argument("--pd", required=True, help="summary JSON (a list takes its first entry)")
    c.add_argument("--out", default=None)
    q = sub.add_parser("policies", help="routing policies side by side, each over round_robin")
    q.add_argument("--summaries", nargs="+", required=True, help="summary JSON files (a list or one summary each)")
    q.add_argument("--baseline", default="round_robin")
    q.add_argument("--out", default=None)
    q.add_argument("--markdown", default=None)
    k = sub.add_parser("correctness", help="per-request token equality of two runs' rows")
    k.add_argument("--left", required=True)
    k.add_argument("--right", required=True)
    k.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    if a.cmd == "single":
        from ...llm import LLM
        from .pairs import load_rows, synthetic_rows
        from ...models.configs import resolve_arch
        llm = LLM(a.model, device=a.device, dtype=a.dtype, max_model_len=a.max_model_len, block_size=a.block_size)
        vocab = resolve_arch(a.model).vocab_size
        if a.dataset:
            rows = load_rows(a.dataset, a.num_requests + a.warmup)
        else:
            rows = synthetic_rows(a.num_requests + a.warmup, a.input_mean, a.output_mean, vocab=vocab)
        res, out = run_single(llm, rows, a.concurrency, a.rate, a.warmup)
        res.update(model=a.model, device=a.device, dtype=a.dtype)
        if a.out:
            Path(a.out).write_text(json.dumps(res, indent=1))
            write_rows(a.out + ".jsonl", out)
    elif a.cmd == "compare":
        single = json.loads(Path(a.single).read_text())
        pd = json.loads(Path(a.pd).read_text())
        res = compare_summaries(single[0] if isinstance(single, list) else single, pd[0] if isinstance(pd, list) else pd)
    elif a.cmd == "policies":
        sums = []
        for path in a.summaries:
            x = json.loads(Path(path).read_text())
            sums += x if isinstance(x, list) else [x]
        res = policy_report(sums, a.baseline)
        if a.markdown:
            Path(a.markdown).write_text(markdown_table(res))
    else:
        res = check_correctness(read_rows(a.left), read_rows(a.right))
    print(json.dumps(res))
    if a.cmd != "single" and a.out:
        Path(a.out).write_text(json.dumps(res, indent=1))
    if a.cmd == "correctness" and not res["passed"]:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
