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
