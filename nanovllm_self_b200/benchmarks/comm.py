"""Tensor-parallel all-reduce + residual + RMSNorm: the fused peer-memory kernel against NCCL.

Launch one process per GPU::

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        -m nanovllm_self_b200.benchmarks.comm [--gemm]

``--gemm`` times the whole row-parallel GEMM + reduction + norm per call instead (see
``main_gemm``), the GEMM -> reduce-scatter path against the all-reduce kernel and NCCL.

For each token count T (hidden 4096, bf16) every variant is captured 20 times into one
CUDA graph and replayed; the time per call is the device time of the replays divided by the
call count, max over ranks.  Variants: ``fused`` (the symmetric-memory kernel: all-reduce,
residual add and RMSNorm in one launch), ``nccl_plus_norm`` (NCCL all_reduce followed by the
fused add + RMSNorm kernel, the baseline), ``norm_only`` (that kernel alone: launch floor).
``roofline_us`` is the NVLink time of the bytes one rank must move for the algorithm the fused
path picks (one-shot: (N-1) T H 2 read; two-shot: 2 (N-1)/N T H 2) at 770 GB/s per direction.
"""
from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist

from ..ops.cuda_ops import CudaOps
from ..parallel.state import init_tensor_parallel
from ..parallel.symm import SymmetricWorkspace

LINK_GBS = 770.0  # measured peer copy bandwidth per direction on this pool's NVSwitch
CALLS = 20


def _graph_time(fn, device) -> float:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    dist.barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(CALLS):
            fn()
    torch.cuda.synchronize()
    dist.barrier()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / (5 * CALLS) * 1e3], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g
    return t.item()


def main(hidden: int = 4096, tokens=(1, 16, 64, 256, 512, 1024, 4096)):
    tp = init_tensor_parallel(int(os.environ["WORLD_SIZE"]), "cuda")
    ops = CudaOps()
    symm = SymmetricWorkspace(tp, rows=max(tokens), hidden=hidden)
    w = torch.ones(hidden, device=tp.device, dtype=torch.bfloat16)
    for T in tokens:
        h = torch.randn(T, hidden, device=tp.device, dtype=torch.bfloat16)
        hh, rr = h.clone(), h.clone()

        def fused():
            return symm.allreduce_add_rmsnorm(symm.input_buffer(T), symm.RES[:T], w, 1e-6, ops)

        def nccl():
            dist.all_reduce(hh)
            return ops.add_rmsnorm(hh, rr, w, 1e-6)

        def norm_only():
            return ops.add_rmsnorm(hh, rr, w, 1e-6)

        tf, tn, t0 = _graph_time(fused, tp.device), _graph_time(nccl, tp.device), _graph_time(norm_only, tp.device)
        one = symm._oneshot(T)
        nbytes = (tp.size - 1) * T * hidden * 2 if one else 2 * (tp.size - 1) / tp.size * T * hidden * 2
        roof = nbytes / (LINK_GBS * 1e3)
        if tp.rank == 0:
            print(json.dumps({"world": tp.size, "T": T, "algo": "one-shot" if one else "two-shot",
                              "fused_us": round(tf, 2), "nccl_plus_norm_us": round(tn, 2), "norm_only_us": round(t0, 2),
                              "roofline_us": round(roof, 2), "frac_roofline": round(roof / tf, 3),
                              "error_word": symm.error()}), flush=True)
    symm.close()
    dist.barrier()
    dist.destroy_process_group()


def main_gemm(hidden: int = 4096, inter: int = 12288, heads: int = 32, tokens=(1, 16, 64, 128, 256)):
    """Row-parallel GEMM + reduction + residual + RMSNorm, per call, for Qwen3-8B's o_proj and down_proj.

    Variants: ``gemm_rs`` (the reduce-scatter in the GEMM epilogue, then the owner-side sum +
    norm + all-gather kernel: the product path for decode steps), ``gemm_allreduce`` (GEMM into
    the symmetric buffer, then the all-reduce + norm kernel), ``gemm_nccl`` (GEMM, NCCL
    all_reduce, add + RMSNorm kernel: the reference's structure) and ``gemm_only`` (no
    reduction).  The weights rotate over enough copies to exceed the L2, as in a forward pass.
    ``roofline_us`` = max(weight bytes / HBM, FLOPs / bf16 peak, NVLink bytes / link) with the
    NVLink bytes of reduce-scatter + all-gather, 2 (N-1)/N T H 2 per rank.
    """
    tp = init_tensor_parallel(int(os.environ["WORLD_SIZE"]), "cuda")
    ops = CudaOps()
    symm = SymmetricWorkspace(tp, rows=max(tokens), hidden=hidden)
    dev = tp.device
    wn = torch.ones(hidden, device=dev, dtype=torch.bfloat16)
    peaks = _peaks()
    for name, k in (("o_proj", heads * 128 // tp.size), ("down_proj", inter // tp.size)):
        wbytes = hidden * k * 2
        copies = max(2, min(CALLS, (256 << 20) // wbytes + 1))
        ws = [(torch.randn(hidden, k, device=dev) * 0.02).to(torch.bfloat16) for _ in range(copies)]
        for T in tokens:
            x = torch.randn(T, k, device=dev).to(torch.bfloat16)
            # residual stream for the reduce-scatter path (its owner rows live in RES)
            symm.allreduce_add_rmsnorm(symm.input_buffer(T), None, wn, 1e-6, ops)
            hh = torch.empty(T, hidden, device=dev, dtype=torch.bfloat16)
            rr = torch.randn(T, hidden, device=dev).to(torch.bfloat16)
            it = [0]

            def nxt():
                it[0] = (it[0] + 1) % copies
                return ws[it[0]]

            def gemm_rs():
                symm.linear_rs(x, nxt(), ops)
                return symm.rs_add_rmsnorm(T, wn, 1e-6, ops)

            def gemm_allreduce():
                ops.linear(x, nxt(), out=symm.input_buffer(T))
                return symm.allreduce_add_rmsnorm(symm.input_buffer(T), symm.RES[:T], wn, 1e-6, ops)

            def gemm_nccl():
                ops.linear(x, nxt(), out=hh)
                dist.all_reduce(hh)
                return ops.add_rmsnorm(hh, rr, wn, 1e-6)

            def gemm_only():
                return ops.linear(x, nxt(), out=hh)

            times = {f.__name__: _graph_time(f, dev) for f in (gemm_rs, gemm_allreduce, gemm_nccl, gemm_only)}
            link = 2 * (tp.size - 1) / tp.size * T * hidden * 2 / (LINK_GBS * 1e3)
            hbm = wbytes / (peaks["hbm_gbs"] * 1e3)
            mma = 2 * T * hidden * k / (peaks["bf16_tflops"] * 1e6)
            roof = max(link, hbm, mma)
            if tp.rank == 0:
                print(json.dumps({"world": tp.size, "op": name, "T": T, "k": k,
                                  **{f"{n}_us": round(t, 2) for n, t in times.items()},
                                  "roofline_us": round(roof, 2), "link_us": round(link, 2), "hbm_us": round(hbm, 2),
                                  "frac_roofline_rs": round(roof / times["gemm_rs"], 3),
                                  "error_word": symm.error()}), flush=True)
    symm.close()
    dist.barrier()
    dist.destroy_process_group()


def _peaks() -> dict:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"])}
    except (OSError, ValueError, KeyError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


if __name__ == "__main__":
    import sys
    if "--gemm" in sys.argv:
        main_gemm()
    else:
        main()
