"""Benchmark drivers for the BASELINE configs (reference ``scripts/benchmark_*.py``).

``python -m nanovllm_self_b200.benchmarks.runners <name> [options]`` with ``name`` in:

* ``runtime``      - TTFT, ITL/TPOT, prefill and decode tok/s for a batch (``benchmark_runtime.py``);
* ``decode_sweep`` - decode tok/s at batch sizes 1/8/32/128/256 with a fixed context (config 3);
* ``kv_dtype``     - the same workload with bf16 and fp8 KV caches (``benchmark_kv_cache_dtype.py``);
* ``prefix``       - the multi-turn agent prefix workload (config 4): prefix-hit rate and tok/s;
* ``pd``           - P/D pool with Poisson arrivals (config 5): p50/p99 TTFT and TPOT;
* ``graph_matrix`` - decode with CUDA graphs against eager decode per batch size, with the graph bucket
  each batch lands in (``benchmark_cuda_graph_matrix.py``, ``_compare.py``, ``_exact_buckets.py``);
* ``mixed``        - mixed-length / shared-prefix regression: greedy outputs against the dense oracle for
  every prefill-attention kernel x CUDA-graph combination, prefix-block reuse checked
  (``benchmark_p0_mixed_workload.py``);
* ``prefill_matrix`` - TTFT, prefill and decode tok/s per prompt length x batch for every prefill-attention
  kernel x CUDA-graph combination, with each combination's gain over the mma.sync kernel without graphs
  (``benchmark_prefill_backends.py``, ``benchmark_prefill_graph_matrix.py``);
* ``decode_vs_hf`` - this engine against the HuggingFace ``generate`` loop on the same random checkpoint
  (``benchmark_decode.py``).
Every driver prints one JSON line (rank 0 under ``torch.distributed.run`` for ``--tp`` > 1), with the
SM clocks and throttle reasons sampled during its timed part.  Warm-up runs use different prompt
token ids than the timed runs (same lengths), so no timed prefill is served from the prefix cache;
the line reports the timed prefix-cache hits.
"""
from __future__ import annotations

import argparse
import json
import os
import time

import torch

from .. import LLM, SamplingParams
from ..utils.clocks import ClockSampler
from . import datasets

WARMUP_SEED = 10_000  # added to a workload's seed for its warm-up copy (same lengths, other token ids)


def _fresh(rows, vocab, seed):
    """Same lengths as `rows`, new token ids."""
    import numpy as np
    rng = np.random.default_rng(seed)
    return [dict(r, prompt_ids=rng.integers(0, vocab, len(r["prompt_ids"])).tolist()) for r in rows]


class _Timed:
    """Clock samples and prefix-cache hits over one timed region."""

    def __init__(self, llm):
        self.llm = llm

    def __enter__(self):
        dev = self.llm.model_runner.device
        self.clk = ClockSampler(dev.index or 0 if dev.type == "cuda" else 0)
        self.hits0 = self.llm.block_manager.num_prefix_hit_blocks
        self.clk.start()
        return self

    def __exit__(self, *a):
        self.clocks = self.clk.stop()
        self.prefix_hits = self.llm.block_manager.num_prefix_hit_blocks - self.hits0


def _llm(args, **kw):
    base = dict(device=args.device, max_model_len=args.max_model_len, max_num_seqs=args.max_num_seqs,
                block_size=args.block_size, kv_cache_quant_mode=args.kv, tensor_parallel_size=args.tp)
    base.update(kw)
    return LLM(args.model, **base)


def _sp(rows):
    return [SamplingParams(temperature=0.0, max_tokens=r["max_tokens"], ignore_eos=True) for r in rows]


def runtime(args) -> dict:
    llm = _llm(args)
    vocab = llm.model_runner.arch.vocab_size
    rows = datasets.uniform_serving(args.batch, vocab, (args.prompt_len, args.prompt_len), (args.gen, args.gen))
    warm = _fresh(rows, vocab, WARMUP_SEED)
    llm.generate([r["prompt_ids"] for r in warm], _sp(warm))
    with _Timed(llm) as t:
        m = llm.generate([r["prompt_ids"] for r in rows], _sp(rows), return_metrics=True)["metrics"]
    prefill_s = m["ttft_ms_p50"] / 1e3
    return {"bench": "runtime", "model": args.model, "tp": args.tp, "batch": args.batch,
            "prompt_len": args.prompt_len, "gen": args.gen,
            "ttft_ms": m["ttft_ms_p50"], "itl_ms": m["tpot_ms_p50"],
            "prefill_tok_s": args.batch * args.prompt_len / prefill_s if prefill_s > 0 else 0.0,
            "decode_tok_s": args.batch / (m["tpot_ms_p50"] / 1e3) if m["tpot_ms_p50"] > 0 else 0.0,
            "e2e_tok_s": m["e2e_throughput_tok_s"], "device_tok_s": m["throughput_tok_s"],
            "prefix_hit_blocks_timed": t.prefix_hits, "clocks": t.clocks}


def decode_sweep(args) -> dict:
    llm = _llm(args)
    vocab = llm.model_runner.arch.vocab_size
    out = {"bench": "decode_sweep", "model": args.model, "tp": args.tp, "context": args.context, "kv": args.kv,
           "gen": args.gen, "points": []}
    for bs in [int(b) for b in args.batches.split(",")]:
        rows = datasets.uniform_serving(bs, vocab, (args.context, args.context), (args.gen, args.gen), seed=bs)
        warm = _fresh(rows, vocab, WARMUP_SEED + bs)
        llm.generate([r["prompt_ids"] for r in warm], _sp(warm))
        with _Timed(llm) as t:
            m = llm.generate([r["prompt_ids"] for r in rows], _sp(rows), return_metrics=True)["metrics"]
        # the decode rate at this batch: device time of the decode-only steps that ran the whole
        # batch (TPOT also counts the prefill steps of later requests that interleave with them)
        n_full, ms_full = m["decode_steps"].get(bs, [0, 0.0])
        out["points"].append({"batch": bs, "decode_step_ms": ms_full, "decode_steps_timed": n_full,
                              "decode_tok_s": bs / (ms_full / 1e3) if ms_full > 0 else 0.0,
                              "tpot_ms_p50": m["tpot_ms_p50"], "ttft_ms_p50": m["ttft_ms_p50"],
                              "prefix_hit_blocks_timed": t.prefix_hits, "clocks": t.clocks})
    return out


def kv_dtype(args) -> dict:
    res = {"bench": "kv_dtype", "runs": []}
    for kv in ("none", "fp8"):
        args.kv = kv
        llm = _llm(args)
        vocab = llm.model_runner.arch.vocab_size
        rows = datasets.uniform_serving(args.batch, vocab, (100, 1024), (100, 1024))
        warm = _fresh(rows, vocab, WARMUP_SEED)
        llm.generate([r["prompt_ids"] for r in warm], _sp(warm))
        with _Timed(llm) as t:
            m = llm.generate([r["prompt_ids"] for r in rows], _sp(rows), return_metrics=True)["metrics"]
        res["runs"].append({"kv": kv, "device_tok_s": m["throughput_tok_s"], "e2e_tok_s": m["e2e_throughput_tok_s"],
                            "tpot_ms": m["tpot_ms_p50"], "kv_blocks": llm.model_runner.num_blocks,
                            "prefix_hit_blocks_timed": t.prefix_hits, "clocks": t.clocks})
        llm.shutdown()
        del llm
        torch.cuda.empty_cache()
    return res


def prefix(args) -> dict:
    llm = _llm(args, enable_chunked_prefill=True, prefill_chunk_size=4096)
    vocab = llm.model_runner.arch.vocab_size
    rows = datasets.agent_sessions(args.sessions, vocab, seed=0)
    by_turn = {}
    for r in rows:
        by_turn.setdefault(r["step_id"], []).append(r)
    # warm-up: one short unrelated batch (compiles graphs, tunes GEMMs; shares no prefix)
    warm = datasets.uniform_serving(4, vocab, (256, 256), (8, 8), seed=WARMUP_SEED)
    llm.generate([r["prompt_ids"] for r in warm], _sp(warm))
    snap0 = llm.block_manager.get_block_usage_snapshot()
    t0 = time.perf_counter()
    gen, dev_s = 0, 0.0
    with _Timed(llm) as tm:
        for t in sorted(by_turn):
            batch = by_turn[t]
            out = llm.generate([r["prompt_ids"] for r in batch], _sp(batch), return_metrics=True)
            gen += out["metrics"]["generated_tokens"]
            dev_s += out["metrics"]["total_time_s"]
    wall = time.perf_counter() - t0
    snap = llm.block_manager.get_block_usage_snapshot()
    hits = snap["prefix_hit_blocks"] - snap0["prefix_hit_blocks"]
    queries = snap["prefix_query_blocks"] - snap0["prefix_query_blocks"]
    return {"bench": "prefix", "model": args.model, "tp": args.tp, "sessions": args.sessions, "turns": len(by_turn),
            "wall_s": wall, "output_tok_s": gen / wall, "device_output_tok_s": gen / dev_s if dev_s else 0.0,
            "prefix_hit_blocks": hits, "prefix_query_blocks": queries, "prefix_hit_rate": hits / max(1, queries),
            "clocks": tm.clocks}


def pd(args) -> dict:
    from ..pd.multiprocess.pool import PDPool
    rows = datasets.pd_lognormal(args.num_requests)
    pool = PDPool(args.work_root, args.num_prefill, args.num_decode, args.pd_backend, args.model,
                  policy="affinity_load_aware", tp=args.tp,
                  worker_args=["--max-model-len", str(args.max_model_len), "--block-size", str(args.block_size),
                               "--kv-cache-quant-mode", args.kv])
    pool.start()
    try:
        s = pool.run(rows, concurrency=None, rate=args.rate)
    finally:
        pool.shutdown()
    s.update(bench="pd", model=args.model, tp_per_worker=args.tp, kv=args.kv, rate=args.rate,
             num_prefill=args.num_prefill, num_decode=args.num_decode, backend=args.pd_backend)
    return s


def graph_matrix(args) -> dict:
    """Decode with CUDA graphs against eager decode, per batch size (one engine of each kind)."""
    from ..engine.model_runner import graph_buckets
    batches = [int(b) for b in args.batches.split(",")]
    graph_max = max(args.max_num_seqs, max(batches))
    buckets = graph_buckets(graph_max)
    timed = {}
    for eager in (False, True):
        llm = _llm(args, enforce_eager=eager, cuda_graph_max_bs=graph_max, max_num_seqs=graph_max)
        vocab = llm.model_runner.arch.vocab_size
        graphs = bool(getattr(llm.model_runner, "graphs", None))
        for bs in batches:
            rows = datasets.uniform_serving(bs, vocab, (args.prompt_len, args.prompt_len), (args.gen, args.gen), seed=bs)
            warm = _fresh(rows, vocab, WARMUP_SEED + bs)
            llm.generate([r["prompt_ids"] for r in warm], _sp(warm))
            with _Timed(llm) as t:
                m = llm.generate([r["prompt_ids"] for r in rows], _sp(rows), return_metrics=True)["metrics"]
            n_full, ms_full = m["decode_steps"].get(bs, [0, 0.0])
            timed[(eager, bs)] = {"graphs_captured": graphs, "decode_step_ms": ms_full, "decode_steps_timed": n_full,
                                  "decode_tok_s": bs / (ms_full / 1e3) if ms_full > 0 else 0.0,
                                  "tpot_ms_p50": m["tpot_ms_p50"], "e2e_tok_s": m["e2e_throughput_tok_s"],
                                  "prefix_hit_blocks_timed": t.prefix_hits, "clocks": t.clocks}
        llm.shutdown()
        del llm
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
    points = []
    for bs in batches:
        g, e = timed[(False, bs)], timed[(True, bs)]
        bucket = next((b for b in buckets if b >= bs), None)
        points.append({"batch": bs, "bucket": bucket, "bucket_kind": "exact" if bucket == bs else "rounded_up",
                       "graph": g, "eager": e,
                       "graph_speedup": e["decode_step_ms"] / g["decode_step_ms"] if g["decode_step_ms"] > 0 else 0.0})
    return {"bench": "graph_matrix", "model": args.model, "tp": args.tp, "prompt_len": args.prompt_len,
            "gen": args.gen, "points": points}


def _combos(cuda: bool) -> list:
    """(prefill-attention kernel, CUDA graphs) pairs this device runs; the torch ops on CPU."""
    return [(k, g) for k in (("tcgen05", "mma") if cuda else ("torch",)) for g in ((True, False) if cuda else (False,))]


def _gain_pct(base, new, larger_is_better):
    if not base:
        return 0.0
    return (new - base) / base * 100.0 if larger_is_better else (base - new) / base * 100.0


def prefill_matrix(args) -> dict:
    """Per (prompt length, batch): TTFT, prefill tok/s, ITL and decode tok/s under every prefill kernel x
    graph combination (one engine per combination, fresh prompts for warm-up and timed runs), and each
    combination's gain over the baseline combination (mma.sync prefill, eager; the torch ops on CPU)."""
    cuda = str(args.device).startswith("cuda")
    combos = _combos(cuda)
    base_key = "mma_graph_off" if cuda else "torch_graph_off"
    lens = [int(x) for x in args.prompt_lens.split(",")]
    batches = [int(x) for x in args.prefill_batches.split(",")]
    per = {}
    for kernel, graph in combos:
        key = f"{kernel}_graph_{'on' if graph else 'off'}"
        llm = _llm(args, enforce_eager=not graph, **({} if kernel == "torch" else {"prefill_attention": kernel}))
        vocab = llm.model_runner.arch.vocab_size
        for n in lens:
            for b in batches:
                rows = datasets.uniform_serving(b, vocab, (n, n), (args.gen, args.gen), seed=31 * n + b)
                warm = _fresh(rows, vocab, WARMUP_SEED + 31 * n + b)
                llm.generate([r["prompt_ids"] for r in warm], _sp(warm))
                with _Timed(llm) as t:
                    m = llm.generate([r["prompt_ids"] for r in rows], _sp(rows), return_metrics=True)["metrics"]
                ttft = m["ttft_ms_p50"]
                per.setdefault((n, b), {})[key] = {
                    "ttft_ms": ttft, "prefill_tok_s": b * n / (ttft / 1e3) if ttft > 0 else 0.0,
                    "itl_ms": m["tpot_ms_p50"],
                    "decode_tok_s": b / (m["tpot_ms_p50"] / 1e3) if m["tpot_ms_p50"] > 0 else 0.0,
                    "e2e_tok_s": m["e2e_throughput_tok_s"], "prefix_hit_blocks_timed": t.prefix_hits,
                    "clocks": t.clocks}
        llm.shutdown()
        del llm
        if cuda:
            torch.cuda.empty_cache()
    cases = []
    for (n, b), by in per.items():
        base = by[base_key]
        gains = {k: {"ttft_gain_pct": _gain_pct(base["ttft_ms"], v["ttft_ms"], False),
                     "decode_gain_pct": _gain_pct(base["decode_tok_s"], v["decode_tok_s"], True)}
                 for k, v in by.items() if k != base_key}
        cases.append({"prompt_len": n, "batch": b, "gen": args.gen, "combos": by, "gain_vs_" + base_key: gains})
    return {"bench": "prefill_matrix", "model": args.model, "tp": args.tp, "baseline": base_key, "cases": cases}


def _first_divergence(model, prompt, got, want):
    """(index, oracle logit gap between its token and the engine's) of the first differing token."""
    from ..models.reference import dense_logits
    for i, (a, b) in enumerate(zip(got, want)):
        if a != b:
            ref = dense_logits(model, list(prompt) + list(got[:i]))
            return i, float((ref[b] - ref[a]).item())
    return None, 0.0


def mixed(args) -> dict:
    """Greedy outputs of mixed-length batches against the dense oracle, for every prefill-attention
    kernel x CUDA-graph combination, and prefix-block reuse of a request sharing a long prefix."""
    from ..models.reference import greedy_generate
    cuda = str(args.device).startswith("cuda")
    gen = args.gen
    combos = _combos(cuda)
    results, oracle = [], {}
    for kernel, graph in combos:
        llm = _llm(args, enforce_eager=not graph, **({} if kernel == "torch" else {"prefill_attention": kernel}))
        runner = llm.model_runner
        vocab, bs = runner.arch.vocab_size, runner.block_size
        g = torch.Generator().manual_seed(7)
        rand = lambda n: torch.randint(0, vocab, (n,), generator=g).tolist()  # noqa: E731
        short = rand(24)
        prefix = rand(2 * bs + 37)
        cases = {"single_short": [short], "mixed_pair": [rand(9), rand(61)], "batch8_short": [short] * 8}
        sp = SamplingParams(temperature=0.0, max_tokens=gen, ignore_eos=True)
        for name, prompts in cases.items():
            t0 = time.perf_counter()
            outs = [o[len(p):] for o, p in zip(llm.generate(prompts, sp), prompts)]
            wall = time.perf_counter() - t0
            rows = []
            for p, o in zip(prompts, outs):
                key = tuple(p)
                if key not in oracle:
                    oracle[key] = greedy_generate(runner.model, p, gen) if args.tp == 1 else None
                want = oracle[key]
                idx, gap = _first_divergence(runner.model, p, o, want) if want is not None else (None, 0.0)
                rows.append({"match": want == o if want is not None else None, "first_divergence": idx,
                             "oracle_gap_at_divergence": gap})
            results.append({"kernel": kernel, "cuda_graph": graph, "case": name, "batch": len(prompts), "gen": gen,
                            "tok_s": len(prompts) * gen / wall, "rows": rows})
        # shared long prefix: the second request must reuse every full block of the prefix
        a, b = prefix + rand(17), prefix + rand(23)
        llm.generate([a], sp)
        hits0 = llm.block_manager.num_prefix_hit_blocks
        out_b = llm.generate([b], sp)[0][len(b):]
        hits = llm.block_manager.num_prefix_hit_blocks - hits0
        if tuple(b) not in oracle:
            oracle[tuple(b)] = greedy_generate(runner.model, b, gen) if args.tp == 1 else None
        want = oracle[tuple(b)]
        idx, gap = _first_divergence(runner.model, b, out_b, want) if want is not None else (None, 0.0)
        results.append({"kernel": kernel, "cuda_graph": graph, "case": "shared_prefix", "batch": 1, "gen": gen,
                        "prefix_hit_blocks": hits, "expected_hit_blocks": len(prefix) // bs,
                        "rows": [{"match": want == out_b if want is not None else None, "first_divergence": idx,
                                  "oracle_gap_at_divergence": gap}]})
        llm.shutdown()
        del llm
        if cuda:
            torch.cuda.empty_cache()
    return {"bench": "mixed", "model": args.model, "tp": args.tp, "block_size": args.block_size, "results": results}


def decode_vs_hf(args) -> dict:
    """This engine against the HuggingFace generate loop, greedy, on one seeded random checkpoint."""
    import tempfile
    from .. import HFLLM
    from ..models.configs import PRESETS
    from ..models.loader import has_checkpoint, save_hf_checkpoint
    arch = PRESETS[args.model]
    path = args.checkpoint or os.path.join(tempfile.gettempdir(), f"nvb_hf_{args.model}_seed0")
    if not has_checkpoint(path):
        save_hf_checkpoint(arch, path, seed=0)
    rows = datasets.uniform_serving(args.batch, arch.vocab_size, (args.prompt_len, args.prompt_len),
                                    (args.gen, args.gen))
    prompts = [r["prompt_ids"] for r in rows]
    sp = SamplingParams(temperature=0.0, max_tokens=args.gen, ignore_eos=True)
    llm = LLM(path, device=args.device, max_model_len=args.max_model_len, max_num_seqs=args.max_num_seqs,
              block_size=args.block_size)
    llm.generate([r["prompt_ids"] for r in _fresh(rows, arch.vocab_size, WARMUP_SEED)], sp)
    t0 = time.perf_counter()
    res = llm.generate(prompts, sp, return_metrics=True)
    ours_s = time.perf_counter() - t0
    ours = [o[len(p):] for o, p in zip(res["outputs"], prompts)]
    llm.shutdown()
    del llm
    hf = HFLLM(path, device=args.device, eos_token_id=-1)
    ids = torch.tensor(prompts, dtype=torch.long)
    hf.generate(ids[:, :8], max_token=2, temperature=0.0)  # warm-up
    if str(args.device).startswith("cuda"):
        torch.cuda.synchronize()
    t0 = time.perf_counter()
    out = hf.generate(ids, max_token=args.gen, temperature=0.0)
    if str(args.device).startswith("cuda"):
        torch.cuda.synchronize()
    hf_s = time.perf_counter() - t0
    theirs = out[:, ids.shape[1]:].tolist()
    first = sum(a[:1] == b[:1] for a, b in zip(ours, theirs)) / len(ours)
    agree = [next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), len(a)) for a, b in zip(ours, theirs)]
    n = args.batch * args.gen
    return {"bench": "decode_vs_hf", "model": args.model, "batch": args.batch, "prompt_len": args.prompt_len,
            "gen": args.gen, "ours_tok_s": n / ours_s, "ours_device_tok_s": res["metrics"]["throughput_tok_s"],
            "hf_tok_s": n / hf_s, "speedup": hf_s / ours_s, "first_token_agreement": first,
            "mean_agreeing_prefix_tokens": sum(agree) / len(agree)}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("name", choices=["runtime", "decode_sweep", "kv_dtype", "prefix", "pd", "graph_matrix", "mixed",
                                     "prefill_matrix", "decode_vs_hf"])
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--kv", default="none")
    ap.add_argument("--max-model-len", type=int, default=9216)
    ap.add_argument("--max-num-seqs", type=int, default=256)
    ap.add_argument("--block-size", type=int, default=256)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--gen", type=int, default=64)
    ap.add_argument("--context", type=int, default=2048)
    ap.add_argument("--batches", default="1,8,32,128,256")
    ap.add_argument("--prompt-lens", default="128,512,2048", help="prefill_matrix: prompt lengths")
    ap.add_argument("--prefill-batches", default="1,8", help="prefill_matrix: batch sizes")
    ap.add_argument("--sessions", type=int, default=64)
    ap.add_argument("--num-requests", type=int, default=512)
    ap.add_argument("--rate", type=float, default=8.0)
    ap.add_argument("--num-prefill", type=int, default=1)
    ap.add_argument("--num-decode", type=int, default=1)
    ap.add_argument("--pd-backend", default="ipc_push")
    ap.add_argument("--work-root", default="/tmp/nvb_pd")
    ap.add_argument("--checkpoint", default=None, help="decode_vs_hf: HF checkpoint directory (written if empty)")
    args = ap.parse_args(argv)
    if args.name == "pd":
        # the pool launches its own worker processes (TP groups via torchrun): run it from one process
        print(json.dumps(pd(args)), flush=True)
        return
    res = globals()[args.name](args)
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
