"""Synthetic workload generators (reference ``scripts/prepare_*_dataset.py``).

* :func:`uniform_serving` - the headline workload: n requests, prompt and output lengths
  uniform in a range, uniform-random token ids;
* :func:`length_matrix` - profiles over a (short/medium/long) x (short/long) grid
  (reference ``prepare_synthetic_serving_dataset.py``);
* :func:`sharegpt_first_turns` - first user turn of each ShareGPT conversation from a local
  JSON file, classified into the same profiles (reference ``prepare_sharegpt_serving_dataset.py``);
* :func:`agent_sessions` - multi-turn agent sessions that share a system prefix, with
  ``program_id`` / ``step_id`` (reference ``prepare_agent_trace_dataset.py``; BASELINE
  config 4: 64 sessions, one 4096-token prefix, 4 turns of lognormal(512, 0.6) appends,
  128 output tokens per turn).
All generators are seeded and return plain dict rows (``prompt_ids``, ``max_tokens`` ...).

From the shell, each generator writes its rows as JSON lines plus a summary (row count, token
totals and percentiles, rows per profile / session)::

    python -m nanovllm_self_b200.benchmarks.datasets synthetic --per-profile 50 --out synth.jsonl
    python -m nanovllm_self_b200.benchmarks.datasets sharegpt --input sg.json --model-path <ckpt> --out sg.jsonl
    python -m nanovllm_self_b200.benchmarks.datasets agent --sessions 64 --out agent.jsonl
    python -m nanovllm_self_b200.benchmarks.datasets uniform|pd --num-requests 256 --out rows.jsonl
"""
from __future__ import annotations

import json

import numpy as np

PROFILES = {"short_short": ((32, 128), (16, 64)), "short_long": ((32, 128), (256, 512)),
            "medium_short": ((256, 768), (16, 64)), "medium_long": ((256, 768), (256, 512)),
            "long_short": ((1024, 3072), (16, 64)), "long_long": ((1024, 3072), (256, 512))}


def uniform_serving(n: int, vocab: int, in_range=(100, 1024), out_range=(100, 1024), seed: int = 0) -> list:
    rng = np.random.default_rng(seed)
    rows = []
    for i in range(n):
        li = int(rng.integers(in_range[0], in_range[1] + 1))
        lo = int(rng.integers(out_range[0], out_range[1] + 1))
        rows.append({"id": f"u{i}", "prompt_ids": rng.integers(0, vocab, li).tolist(), "max_tokens": lo,
                     "input_tokens": li})
    return rows


def classify(input_tokens: int, output_tokens: int) -> str:
    a = "short" if input_tokens < 256 else "medium" if input_tokens < 1024 else "long"
    b = "short" if output_tokens < 128 else "long"
    return f"{a}_{b}"


def length_matrix(per_profile: int, vocab: int, seed: int = 0, profiles=None) -> list:
    rng = np.random.default_rng(seed)
    rows = []
    for name in (profiles or PROFILES):
        (i0, i1), (o0, o1) = PROFILES[name]
        for k in range(per_profile):
            li, lo = int(rng.integers(i0, i1 + 1)), int(rng.integers(o0, o1 + 1))
            rows.append({"id": f"{name}-{k}", "profile": name, "prompt_ids": rng.integers(0, vocab, li).tolist(),
                         "max_tokens": lo, "input_tokens": li})
    return rows


def sharegpt_first_turns(path: str, encode, max_rows: int = 1000, max_tokens: int = 256) -> list:
    with open(path) as f:
        data = json.load(f)
    rows = []
    for conv in data:
        turns = conv.get("conversations") or conv.get("items") or []
        first = next((t for t in turns if t.get("from") in ("human", "user")), None)
        if first is None:
            continue
        ids = encode(first.get("value", ""))
        if not ids:
            continue
        rows.append({"id": conv.get("id", f"sg{len(rows)}"), "prompt_ids": ids, "max_tokens": max_tokens,
                     "input_tokens": len(ids), "profile": classify(len(ids), max_tokens)})
        if len(rows) >= max_rows:
            break
    return rows


def agent_sessions(n_sessions: int = 64, vocab: int = 151936, prefix_len: int = 4096, turns: int = 4,
                   append_mean: float = 512, append_sigma: float = 0.6, output_tokens: int = 128,
                   seed: int = 0) -> list:
    """Rows grouped by session; turn t of a session extends turn t-1's prompt (+ its output
    placeholder) with a new user/tool segment, all behind one shared system prefix."""
    rng = np.random.default_rng(seed)
    prefix = rng.integers(0, vocab, prefix_len).tolist()
    rows = []
    for s in range(n_sessions):
        ctx = list(prefix)
        for t in range(turns):
            n_app = int(max(8, rng.lognormal(np.log(append_mean), append_sigma)))
            ctx = ctx + rng.integers(0, vocab, n_app).tolist()
            rows.append({"id": f"s{s}-t{t}", "program_id": f"sess-{s}", "session_id": f"sess-{s}", "step_id": t,
                         "prompt_ids": list(ctx), "max_tokens": output_tokens, "input_tokens": len(ctx),
                         "task_type": "mixed_agent"})
            # the next turn's prompt contains this turn's answer; ids stand in for it
            ctx = ctx + rng.integers(0, vocab, output_tokens).tolist()
    return rows


def poisson_arrivals(n: int, rate: float, seed: int = 0) -> list:
    rng = np.random.default_rng(seed)
    return np.cumsum(rng.exponential(1.0 / rate, n)).tolist()


def pd_lognormal(n: int, vocab: int = 151936, in_mean=2048, in_sigma=0.5, in_max=8192, out_mean=256, out_sigma=0.5,
                 out_max=1024, seed: int = 0) -> list:
    """BASELINE config 5 lengths: lognormal input (mean 2048, clip 8192) and output (mean 256, clip 1024)."""
    rng = np.random.default_rng(seed)
    rows = []
    for i in range(n):
        li = int(np.clip(rng.lognormal(np.log(in_mean), in_sigma), 16, in_max))
        lo = int(np.clip(rng.lognormal(np.log(out_mean), out_sigma), 4, out_max))
        rows.append({"id": f"pd{i}", "prompt_ids": rng.integers(0, vocab, li).tolist(), "max_tokens": lo,
                     "input_tokens": li})
    return rows


def summarize(rows: list) -> dict:
    """Row count, input / output token totals and percentiles, rows per profile and per session."""
    ins = np.asarray([len(r["prompt_ids"]) for r in rows] or [0])
    outs = np.asarray([r["max_tokens"] for r in rows] or [0])
    pct = lambda a: {f"p{q}": float(np.percentile(a, q)) for q in (50, 90, 99)}  # noqa: E731
    out = {"rows": len(rows), "input_tokens": int(ins.sum()), "output_tokens": int(outs.sum()),
           "input_pct": pct(ins), "output_pct": pct(outs)}
    for key in ("profile", "session_id"):
        if rows and key in rows[0]:
            counts: dict = {}
            for r in rows:
                counts[r[key]] = counts.get(r[key], 0) + 1
            out[f"rows_per_{key}"] = counts
    return out


def main(argv=None) -> dict:
    import argparse
    ap = argparse.ArgumentParser(description="write a benchmark workload as JSON lines plus a summary")
    ap.add_argument("kind", choices=["synthetic", "sharegpt", "agent", "uniform", "pd"])
    ap.add_argument("--out", required=True, help="rows (JSON lines); the summary goes to <out>.summary.json")
    ap.add_argument("--vocab", type=int, default=151936)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--per-profile", type=int, default=50, help="synthetic: rows per length profile")
    ap.add_argument("--input", help="sharegpt: the ShareGPT JSON file")
    ap.add_argument("--model-path", help="sharegpt: checkpoint directory whose tokenizer encodes the turns")
    ap.add_argument("--max-rows", type=int, default=1000)
    ap.add_argument("--max-tokens", type=int, default=256, help="sharegpt / agent: output tokens per row")
    ap.add_argument("--sessions", type=int, default=64)
    ap.add_argument("--turns", type=int, default=4)
    ap.add_argument("--prefix-len", type=int, default=4096)
    ap.add_argument("--num-requests", type=int, default=256)
    a = ap.parse_args(argv)
    if a.kind == "synthetic":
        rows = length_matrix(a.per_profile, a.vocab, a.seed)
    elif a.kind == "sharegpt":
        if not (a.input and a.model_path):
            raise SystemExit("sharegpt needs --input and --model-path (a tokenizer)")
        from transformers import AutoTokenizer
        tok = AutoTokenizer.from_pretrained(a.model_path)
        rows = sharegpt_first_turns(a.input, lambda t: tok(t)["input_ids"], a.max_rows, a.max_tokens)
    elif a.kind == "agent":
        rows = agent_sessions(a.sessions, a.vocab, a.prefix_len, a.turns, output_tokens=a.max_tokens, seed=a.seed)
    elif a.kind == "uniform":
        rows = uniform_serving(a.num_requests, a.vocab, seed=a.seed)
    else:
        rows = pd_lognormal(a.num_requests, a.vocab, seed=a.seed)
    with open(a.out, "w") as f:
        for r in rows:
            f.write(json.dumps(r) + "\n")
    summary = dict(summarize(rows), kind=a.kind, seed=a.seed, path=a.out)
    with open(a.out + ".summary.json", "w") as f:
        json.dump(summary, f, indent=1)
    print(json.dumps({k: v for k, v in summary.items() if not k.startswith("rows_per_session")}))
    return summary


if __name__ == "__main__":
    main()
