"""One engine step of a real model, for timing or for a profiler's per-kernel launch list.

``python -m nanovllm_self_b200.benchmarks.step_profile decode --batch 256 --ctx 600``
``python -m nanovllm_self_b200.benchmarks.step_profile prefill --batch 16 --ctx 1024``

``decode`` builds ``batch`` sequences whose first ``ctx`` tokens are already in the KV cache
(random contents: the step's cost does not depend on them) and runs decode steps through
``ModelRunner.run`` (a CUDA-graph replay when the batch has a bucket); ``prefill`` runs one
prefill step of ``batch`` fresh prompts of ``ctx`` tokens (eager).  Both use random-init
weights of ``--model`` (default Qwen3-8B), TP=1.

``--mode time`` (default) prints one JSON line with the CUDA-event time per step (median of
``--iters``).  ``--mode profile`` runs two warm-up steps, then ONE step between
``cudaProfilerStart``/``cudaProfilerStop``: with
``ncu --profile-from-start off --metrics gpu__time_duration.sum --clock-control none`` this gives
the device time of every kernel of one step (one pass per kernel).
"""
from __future__ import annotations

import argparse
import json
import statistics

import numpy as np
import torch


def _engine(model: str, batch: int, ctx: int, kv: str):
    from nanovllm_self_b200 import LLM
    blocks = batch * ((ctx + 64 + 255) // 256) + 8  # just the step's KV: a small device footprint
    return LLM(model, device="cuda:0", max_model_len=ctx + 64, max_num_seqs=max(batch, 1),
               max_num_batched_tokens=max(16384, batch * ctx), block_size=256, cuda_graph_max_bs=max(batch, 1),
               num_blocks=blocks, kv_cache_quant_mode="fp8" if kv == "fp8" else "none")


def _decode_seqs(llm, batch: int, ctx: int):
    from nanovllm_self_b200.engine.sequence import Sequence
    from nanovllm_self_b200.sampling_params import SamplingParams
    r = llm.model_runner
    rng = np.random.default_rng(0)
    seqs = []
    for i in range(batch):
        s = Sequence(i, rng.integers(0, r.arch.vocab_size, size=ctx).tolist(),
                     SamplingParams(temperature=0.0, max_tokens=1 << 20, ignore_eos=True), r.block_size)
        r.block_manager.allocate(s)
        s.append_token(int(rng.integers(0, r.arch.vocab_size)))
        s.num_cached_tokens = ctx
        s.num_new_tokens = 1
        if len(s.block_table) * r.block_size < ctx + 1:
            r.block_manager.may_append(s)
        seqs.append(s)
    return seqs


def _prefill_seqs(llm, batch: int, ctx: int, seed: int):
    from nanovllm_self_b200.engine.sequence import Sequence
    from nanovllm_self_b200.sampling_params import SamplingParams
    r = llm.model_runner
    rng = np.random.default_rng(seed)
    seqs = []
    for i in range(batch):
        s = Sequence(seed * 100000 + i, rng.integers(0, r.arch.vocab_size, size=ctx).tolist(),
                     SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True), r.block_size)
        r.block_manager.allocate(s)
        s.num_new_tokens = ctx - s.num_cached_tokens
        seqs.append(s)
    return seqs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kind", choices=["decode", "prefill"])
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--ctx", type=int, default=600)
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--kv", choices=["bf16", "fp8"], default="bf16")
    ap.add_argument("--mode", choices=["time", "profile"], default="time")
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args()
    llm = _engine(a.model, a.batch, a.ctx, a.kv)
    r = llm.model_runner
    bm = r.block_manager

    def step(i):
        if a.kind == "decode":
            return r.run(seqs)
        ps = _prefill_seqs(llm, a.batch, a.ctx, seed=i + 1)
        out = r.run(ps)
        for s in ps:
            bm.deallocate(s)
        return out

    seqs = _decode_seqs(llm, a.batch, a.ctx) if a.kind == "decode" else None
    for i in range(2):
        step(i)
    torch.cuda.synchronize()
    if a.mode == "profile":
        torch.cuda.profiler.start()
        step(2)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"kind": a.kind, "batch": a.batch, "ctx": a.ctx, "profiled_steps": 1}))
        return
    times = []
    for i in range(a.iters):
        step(3 + i)
        times.append(r.last_dev_ms)
    tokens = a.batch if a.kind == "decode" else a.batch * a.ctx
    med = statistics.median(times)
    print(json.dumps({"kind": a.kind, "model": a.model, "kv": a.kv, "batch": a.batch, "ctx": a.ctx,
                      "step_ms": round(med, 3), "tokens_per_s": round(tokens / (med / 1e3), 1),
                      "graph": a.kind == "decode" and r.enable_cuda_graph}))


if __name__ == "__main__":
    main()
