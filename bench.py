"""Headline benchmark: offline output tokens/s of Qwen3-8B (random init, bf16) at TP = N.

Workload (BASELINE config 2/3): 256 requests, prompt lengths uniform in [100, 1024],
output lengths uniform in [100, 1024], uniform-random prompt token ids, greedy,
ignore_eos; paged KV with block 256; CUDA-graph decode buckets.

One "step" is one complete ``LLM.generate`` over the 256 requests (prefill + decode
until every request finishes).  Every warm-up and timed step draws fresh prompt token
ids (same lengths), so no prefill is served from the prefix cache; the JSON line
reports the timed prefix-cache hits (``prefix_hit_blocks_timed``, expected 0).  W warm-up steps, then exactly K timed steps bracketed
by a barrier and ``torch.cuda.synchronize()`` on both sides.

* ``value``: generated tokens / summed device time of the engine steps (CUDA events
  around each forward + sample), max over ranks: what the kernels take.
* ``e2e.value``: generated tokens / CUDA-event time of the whole ``generate`` call,
  max over ranks: host scheduling, input packing, the pinned host-to-device copy of
  every engine step's inputs and the device-to-host copy of its sampled ids included.

``--impl reference`` runs the unmodified reference (``baseline/_ref``) through its own
public API on the same workload, or prints an ``unavailable`` line.

Launch: ``python bench.py`` (1 GPU) or ``python -m torch.distributed.run --nproc-per-node N
--master-addr 127.0.0.1 --master-port P bench.py --gpus N``.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from nanovllm_self_b200.utils.clocks import ClockSampler  # noqa: E402

METRIC = "output tok/s (device-timed, max over ranks) Qwen3-8B TP1/2/4/8; p50 TTFT/TPOT"
MODEL_NAMES = {"qwen3-8b": "Qwen3-8B", "qwen3-0.6b": "Qwen3-0.6B", "qwen3-32b": "Qwen3-32B"}


def workload(n: int, vocab: int, seed: int = 0, in_range=(100, 1024), out_range=(100, 1024), token_seed=None):
    """`n` requests: lengths drawn from `seed`, prompt token ids from `token_seed` (default `seed`).

    Every benchmark step passes its own `token_seed`, so no step repeats another step's prompts
    and no prefill is served from the prefix cache; the lengths, and so the work, stay the same.
    """
    import numpy as np
    rng = np.random.default_rng(seed)
    ins = rng.integers(in_range[0], in_range[1] + 1, size=n)
    outs = rng.integers(out_range[0], out_range[1] + 1, size=n)
    trng = rng if token_seed is None else np.random.default_rng([seed, int(token_seed)])
    prompts = [trng.integers(0, vocab, size=int(l)).tolist() for l in ins]
    return prompts, [int(o) for o in outs]


def step_seed(phase: str, i: int) -> int:
    """Token seed of warm-up step i ("warmup") or timed step i ("timed"); all distinct."""
    return (1 if phase == "warmup" else 2) * 100000 + i


def dist_info():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def reduce_max(vals, world, device):
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def run_ours(args):
    import torch
    import torch.distributed as dist
    from nanovllm_self_b200 import LLM, SamplingParams
    rank, world, local = dist_info()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    device = f"cuda:{local}"
    torch.cuda.set_device(local)
    kv_mode = "fp8" if args.kv == "fp8" else "none"
    llm = LLM(args.model, tensor_parallel_size=args.gpus, device=device, max_model_len=2048 + 64,
              max_num_seqs=256, max_num_batched_tokens=16384, block_size=256, cuda_graph_max_bs=512,
              kv_cache_quant_mode=kv_mode, comm_backend=args.comm)
    vocab = llm.model_runner.arch.vocab_size
    _, outs = workload(args.num_requests, vocab)
    sps = [SamplingParams(temperature=0.0, max_tokens=o, ignore_eos=True) for o in outs]
    for i in range(args.warmup):
        llm.generate(workload(args.num_requests, vocab, token_seed=step_seed("warmup", i))[0], sps)
    timed_prompts = [workload(args.num_requests, vocab, token_seed=step_seed("timed", i))[0]
                     for i in range(args.steps)]
    runner = llm.model_runner
    ops = runner.ops
    bm = llm.block_manager
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = getattr(ops, "launches", 0) + (llm.comm.launches if llm.comm is not None else 0)
    h2d0, d2h0 = runner.h2d_bytes, runner.d2h_bytes
    hits0 = bm.num_prefix_hit_blocks
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    dev_ms = 0.0
    gen = 0
    steps_engine = 0
    ttft, tpot = [], []
    for prompts in timed_prompts:
        res = llm.generate(prompts, sps, return_metrics=True)
        m = res["metrics"]
        dev_ms += m["total_time_s"] * 1e3
        gen += m["generated_tokens"]
        steps_engine += m["schedule_steps"]
        ttft.append(m["ttft_ms_p50"])
        tpot.append(m["tpot_ms_p50"])
    ev1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    wall_ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    launches = getattr(ops, "launches", 0) + (llm.comm.launches if llm.comm is not None else 0) - launches0
    h2d, d2h = runner.h2d_bytes - h2d0, runner.d2h_bytes - d2h0
    prefix_hits = bm.num_prefix_hit_blocks - hits0
    dev_max, wall_max = reduce_max([dev_ms, wall_ms], world, device)
    llm.shutdown()
    if rank == 0:
        name = MODEL_NAMES.get(args.model, args.model)
        value = gen / (dev_max / 1e3)
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(wall_max / args.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: uniform-random prompt token ids, random-init weights N(0, 0.02), seed 0",
            "config": {"model": name, "global_batch": args.num_requests,
                       "seq_len": "prompt U[100,1024], output U[100,1024]",
                       "parallelism": f"tp{args.gpus}", "kv_cache": args.kv, "comm_backend": args.comm,
                       "block_size": 256, "cuda_graph_buckets": "1,2,4,8,16..256",
                       "l2": "no flush: each step streams the full weights (>> 126 MB L2)",
                       "prompts": "fresh token ids every warm-up and timed step (same lengths)",
                       "step": "one LLM.generate over all requests", "engine_steps_per_step": steps_engine
                       // max(args.steps, 1)},
            "prefix_hit_blocks_timed": int(prefix_hits),
            "generated_tokens_per_step": gen // max(args.steps, 1),
            "ttft_ms_p50": round(sum(ttft) / len(ttft), 3), "tpot_ms_p50": round(sum(tpot) / len(tpot), 3),
            "clocks": clk,
            "e2e": {"value": round(gen / (wall_max / 1e3), 2), "unit": "tok/s",
                    "h2d_bytes_per_step": int(h2d // max(args.steps, 1)),
                    "d2h_bytes_per_step": int(d2h // max(args.steps, 1))},
            "gpu_launches": int(launches),
            "impl": "ours",
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_reference(args):
    from baseline_ref import run_reference_arm  # noqa: WPS433 (kept beside bench.py)
    run_reference_arm(args, workload, step_seed, ClockSampler, dist_info, reduce_max, METRIC, MODEL_NAMES)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--kv", choices=["bf16", "fp8"], default="bf16")
    ap.add_argument("--comm", choices=["fused", "nccl"], default="fused")
    ap.add_argument("--num-requests", type=int, default=256)
    args = ap.parse_args()
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
