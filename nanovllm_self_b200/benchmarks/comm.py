"""Tensor-parallel all-reduce + residual + RMSNorm: the fused peer-memory kernel against NCCL.

Launch one process per GPU::

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        -m nanovllm_self_b200.benchmarks.comm

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


if __name__ == "__main__":
    main()
