"""TP consistency and per-rank memory matrix: the same greedy request at TP = 1, 2, 4 (8),
tokens compared against TP = 1, every rank's memory reported.

Reference: ``scripts/run_tp_memory_consistency_matrix.sh`` with ``tests/test_tp_generate.py``
(one prompt, 16 greedy tokens per TP size; rank 0 gathers each rank's
``memory_allocated`` / ``max_memory_allocated`` / ``memory_reserved`` and writes
``tp<N>.json``; a summary marks which sizes match TP = 1 and lists the per-rank peaks).

Here each rank reports, besides the CUDA allocator's counters (zero on CPU ranks), the bytes
it holds by owner: its weight shard (:meth:`Qwen3ForCausalLM.weight_bytes`), its KV pool
shard (its KV heads only) and the per-block scales.  The summary adds the check that
sharding actually divides the model: ``weight_shard_ratio`` = TP x the largest rank's weight
bytes / TP = 1's weight bytes (1.0 when everything is sharded; the replicated norms put it a
little above), and the same for the KV pool per block.

Every size and the summary in one command (TP > 1 sizes through ``torch.distributed.run``)::

    python -m nanovllm_self_b200.benchmarks.tp_matrix matrix --result-dir /tmp/tpm --tps 1,2,4 --model qwen3-8b

or one command per size, then the summary::

    python -m nanovllm_self_b200.benchmarks.tp_matrix run --result-dir /tmp/tpm --model qwen3-8b
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m nanovllm_self_b200.benchmarks.tp_matrix \\
        run --result-dir /tmp/tpm --model qwen3-8b
    python -m nanovllm_self_b200.benchmarks.tp_matrix summary --result-dir /tmp/tpm --tps 1,2,4
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path

import torch

MB = 1024.0 * 1024.0


def default_prompt(vocab: int, n: int = 24, seed: int = 0) -> list:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n,), generator=g).tolist()


def rank_memory(llm) -> dict:
    """This rank's bytes by owner, and the CUDA allocator's counters on GPU ranks."""
    mr = llm.model_runner
    kv = mr.kv_cache.numel() * mr.kv_cache.element_size()
    sc = mr.kv_scale_cache
    out = {"rank": mr.tp.rank, "device": str(mr.device), "weight_mb": mr.model.weight_bytes() / MB,
           "kv_cache_mb": kv / MB, "kv_scale_mb": (sc.numel() * sc.element_size() / MB) if sc is not None else 0.0,
           "num_kv_blocks": mr.num_blocks, "kv_heads": mr.model.num_kv_heads,
           "memory_allocated_mb": 0.0, "max_memory_allocated_mb": 0.0, "memory_reserved_mb": 0.0,
           "max_memory_reserved_mb": 0.0}
    if mr.is_cuda:
        out.update(memory_allocated_mb=torch.cuda.memory_allocated() / MB,
                   max_memory_allocated_mb=torch.cuda.max_memory_allocated() / MB,
                   memory_reserved_mb=torch.cuda.memory_reserved() / MB,
                   max_memory_reserved_mb=torch.cuda.max_memory_reserved() / MB)
    return out


def run_case(result_dir, model: str = "qwen3-8b", max_tokens: int = 16, prompt=None, **engine_kw) -> dict | None:
    """One TP size (WORLD_SIZE ranks, this process one of them): greedy tokens and every
    rank's memory; rank 0 writes ``tp<N>.json`` and returns its record."""
    from .. import LLM, SamplingParams
    from ..models.configs import resolve_arch
    tp = int(os.environ.get("WORLD_SIZE", "1"))
    if str(engine_kw.get("device", "cuda")).startswith("cuda"):
        torch.cuda.reset_peak_memory_stats()
    llm = LLM(model, tensor_parallel_size=tp, **engine_kw)
    prompt = prompt if prompt is not None else default_prompt(resolve_arch(model).vocab_size)
    out = llm.generate([prompt], SamplingParams(temperature=0.0, max_tokens=max_tokens, ignore_eos=True))[0]
    mem = rank_memory(llm)
    if tp > 1:
        import torch.distributed as dist
        gathered = [None] * tp
        dist.all_gather_object(gathered, mem)
    else:
        gathered = [mem]
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    rec = {"tp": tp, "model": model, "prompt_tokens": len(prompt), "generated_token_ids": out[len(prompt):],
           "rank_memory": gathered}
    Path(result_dir).mkdir(parents=True, exist_ok=True)
    (Path(result_dir) / f"tp{tp}.json").write_text(json.dumps(rec, indent=1))
    return rec


def summarize(result_dir, tps=(1, 2, 4)) -> dict:
    """Token equality with TP = 1 and the per-rank memory of every size present."""
    rows = {}
    for tp in tps:
        p = Path(result_dir) / f"tp{tp}.json"
        if p.exists():
            rows[tp] = json.loads(p.read_text())
    if 1 not in rows:
        raise FileNotFoundError(f"{result_dir}/tp1.json: the TP = 1 case is the baseline")
    base = rows[1]
    w1 = base["rank_memory"][0]["weight_mb"]
    kv1 = base["rank_memory"][0]["kv_cache_mb"] / max(1, base["rank_memory"][0]["num_kv_blocks"])
    cases = {}
    for tp, r in sorted(rows.items()):
        mem = r["rank_memory"]
        kv_per_block = max(m["kv_cache_mb"] / max(1, m["num_kv_blocks"]) for m in mem)
        cases[str(tp)] = {
            "generated_token_ids": r["generated_token_ids"],
            "matches_tp1": r["generated_token_ids"] == base["generated_token_ids"],
            "ranks": len(mem),
            "weight_mb_per_rank": [round(m["weight_mb"], 3) for m in mem],
            "weight_shard_ratio": tp * max(m["weight_mb"] for m in mem) / w1 if w1 else None,
            "kv_block_shard_ratio": tp * kv_per_block / kv1 if kv1 else None,
            "max_memory_allocated_mb_per_rank": [round(m["max_memory_allocated_mb"], 1) for m in mem],
            "rank_memory": mem,
        }
    summary = {"result_dir": str(result_dir), "baseline_tp": 1, "cases": cases,
               "all_match": all(c["matches_tp1"] for c in cases.values())}
    (Path(result_dir) / "summary.json").write_text(json.dumps(summary, indent=1))
    return summary


RUN_OPTS = ("model", "device", "dtype", "max_tokens", "max_model_len", "block_size", "num_blocks", "kv")


def run_matrix(result_dir, tps, run_argv: list, timeout_s: float = 3600.0, port: int = 29871) -> dict:
    """Each TP size as its own job (TP = 1 in one process, larger sizes under
    ``torch.distributed.run`` on 127.0.0.1), then :func:`summarize`."""
    import subprocess
    import sys
    for tp in tps:
        mod = ["-m", "nanovllm_self_b200.benchmarks.tp_matrix", "run", "--result-dir", str(result_dir), *run_argv]
        if tp > 1:
            cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={tp}",
                   "--master-addr", "127.0.0.1", f"--master-port={port + tp}", *mod]
        else:
            cmd = [sys.executable, *mod]
        subprocess.run(cmd, check=True, timeout=timeout_s)
    return summarize(result_dir, tuple(tps))


def _run_args(p):
    p.add_argument("--model", default="qwen3-8b")
    p.add_argument("--device", default="cuda")
    p.add_argument("--dtype", default="bf16")
    p.add_argument("--max-tokens", type=int, default=16)
    p.add_argument("--max-model-len", type=int, default=4096)
    p.add_argument("--block-size", type=int, default=256)
    p.add_argument("--num-blocks", type=int, default=-1, help="-1 sizes the KV pool from free memory")
    p.add_argument("--kv", default="none", help="kv_cache_quant_mode")


def _print_summary(res) -> None:
    print(json.dumps({tp: {k: c[k] for k in ("matches_tp1", "weight_shard_ratio", "kv_block_shard_ratio",
                                              "max_memory_allocated_mb_per_rank")}
                      for tp, c in res["cases"].items()}))


def main(argv=None):
    ap = argparse.ArgumentParser(description="TP consistency / per-rank memory matrix")
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run", help="one TP size (launch with torchrun for TP > 1)")
    r.add_argument("--result-dir", required=True)
    _run_args(r)
    m = sub.add_parser("matrix", help="every TP size, each as its own job, then the summary")
    m.add_argument("--result-dir", required=True)
    m.add_argument("--tps", default="1,2,4")
    _run_args(m)
    s = sub.add_parser("summary", help="compare the sizes written so far")
    s.add_argument("--result-dir", required=True)
    s.add_argument("--tps", default="1,2,4")
    a = ap.parse_args(argv)
    if a.cmd == "run":
        rec = run_case(a.result_dir, a.model, a.max_tokens, device=a.device, dtype=a.dtype,
                       max_model_len=a.max_model_len, block_size=a.block_size, num_blocks=a.num_blocks,
                       kv_cache_quant_mode=a.kv, comm_backend="nccl" if a.device == "cpu" else "fused")
        if rec is not None:
            print(json.dumps({k: v for k, v in rec.items() if k != "rank_memory"}), flush=True)
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            import torch.distributed as dist
            dist.barrier()
            os._exit(0)  # the group is not torn down at exit: gloo's destructor can race its own threads
        return
    if a.cmd == "matrix":
        run_argv = []
        for k in RUN_OPTS:
            run_argv += [f"--{k.replace('_', '-')}", str(getattr(a, k))]
        res = run_matrix(a.result_dir, [int(x) for x in a.tps.split(",")], run_argv)
        _print_summary(res)
        if not res["all_match"]:
            raise SystemExit(1)
        return
    else:
        res = summarize(a.result_dir, tuple(int(x) for x in a.tps.split(",")))
        _print_summary(res)
        if not res["all_match"]:
            raise SystemExit(1)


if __name__ == "__main__":
    main()
