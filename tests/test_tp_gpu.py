"""Tensor parallelism on 2+ GPUs: fused NVLink all-reduce path vs the NCCL path vs TP=1.

Needs at least two GPUs (skipped otherwise).  Ranks are child processes over NCCL with
NVLS disabled; every device wait in the fused kernel is bounded.
"""
import json
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _prompts():
    g = torch.Generator().manual_seed(5)
    return [torch.randint(0, 151936, (n,), generator=g).tolist() for n in (37, 300, 128, 700)]


def _short_prompts():
    # prompt + 16 generated tokens stay within one decode-sized step (<= 256 rows), so the
    # teacher-forced scoring forward below also takes the GEMM -> reduce-scatter path
    g = torch.Generator().manual_seed(9)
    return [torch.randint(0, 151936, (n,), generator=g).tolist() for n in (37, 100, 128, 200)]


def _score(llm, seq):
    """Teacher-forced logits [len(seq), V] of one sequence (one forward), gathered over the shards."""
    import torch.distributed as dist
    from nanovllm_self_b200.engine.sequence import Sequence
    from nanovllm_self_b200.sampling_params import SamplingParams
    r = llm.model_runner
    s = Sequence(10 ** 6, seq, SamplingParams(temperature=0, max_tokens=1), r.block_size)
    # every position is computed here: no block may come from the prefix cache (the generate
    # call before left this sequence's prefix blocks in it)
    bm = r.block_manager
    saved, bm.enable_prefix_cache = bm.enable_prefix_cache, False
    try:
        bm.allocate(s)
    finally:
        bm.enable_prefix_cache = saved
    assert s.num_cached_tokens == 0
    s.num_new_tokens = len(s.token_ids) - s.num_cached_tokens
    pk = r._pack([s])
    ids, pos, ctx, _, _ = r._to_device(pk)
    ctx.logits_indices = torch.arange(len(seq), device=ids.device, dtype=ctx.logits_indices.dtype)
    with torch.inference_mode():
        part = r.model.forward(ids, pos, ctx, r.kv_layers, r.kv_scale_layers)
    r.block_manager.deallocate(s)
    world = llm.tp.size
    if world == 1:
        return part[:, :r.model.vocab_size].float().cpu()
    parts = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(parts, part.contiguous())
    return torch.cat(parts, dim=1)[:, :r.model.vocab_size].float().cpu()


def _kw(backend):
    """``fused``: one-shot / two-shot all-reduce kernels; ``fused_rs``: decode-sized steps take the
    GEMM -> reduce-scatter path; ``nccl``: the NCCL baseline."""
    kw = dict(max_model_len=2048, max_num_seqs=16, num_blocks=64, cuda_graph_max_bs=16)
    if backend == "fused_rs":
        return dict(kw, comm_backend="fused", fused_reduce_scatter=True)
    return dict(kw, comm_backend=backend)


def _worker(rank, world, port, out_path, backend):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from nanovllm_self_b200 import LLM, SamplingParams
    from nanovllm_self_b200.engine.sequence import Sequence
    llm = LLM("qwen3-0.6b", tensor_parallel_size=world, device=f"cuda:{rank}", **_kw(backend))
    out = llm.generate(_prompts(), SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True))
    # logits of one prefill, gathered over the vocab shards
    r = llm.model_runner
    s = Sequence(0, _prompts()[1], SamplingParams(temperature=0, max_tokens=1), r.block_size)
    r.block_manager.allocate(s)
    s.num_new_tokens = len(s.token_ids) - s.num_cached_tokens
    pk = r._pack([s])
    ids, pos, ctx, _, _ = r._to_device(pk)
    with torch.inference_mode():
        part = r.model.forward(ids, pos, ctx, r.kv_layers, r.kv_scale_layers)
    import torch.distributed as dist
    parts = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(parts, part.contiguous())
    logits = torch.cat(parts, dim=1)[0, :r.model.vocab_size].float().cpu()
    # short prompts: decode steps and the scoring forwards are decode-sized (reduce-scatter path)
    short = llm.generate(_short_prompts(), SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True))
    scores = {"short": [_score(llm, seq) for seq in short], "out": [_score(llm, seq) for seq in out]}
    err = llm.comm.symm.error() if llm.comm.symm is not None else 0
    if rank == 0:
        torch.save({"out": out, "logits": logits, "err": err, "short": short, "scores": scores}, out_path)
    llm.shutdown()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_fused_matches_nccl_and_tp1(tmp_path):
    from nanovllm_self_b200 import LLM
    from nanovllm_self_b200.engine.sequence import Sequence
    from nanovllm_self_b200.sampling_params import SamplingParams
    res = {}
    for backend in ("fused", "fused_rs", "nccl"):
        path = str(tmp_path / f"{backend}.pt")
        mp.spawn(_worker, args=(2, _free_port(), path, backend), nprocs=2, join=True)
        res[backend] = torch.load(path)
    assert res["fused"]["err"] == 0 and res["fused_rs"]["err"] == 0
    lf, ln = res["fused"]["logits"], res["nccl"]["logits"]
    assert torch.nn.functional.cosine_similarity(lf, ln, dim=0).item() > 0.999
    assert torch.nn.functional.cosine_similarity(res["fused_rs"]["logits"], ln, dim=0).item() > 0.999
    llm = LLM("qwen3-0.6b", device="cuda:0", **_kw("nccl"))
    r = llm.model_runner
    s = Sequence(0, _prompts()[1], SamplingParams(temperature=0, max_tokens=1), r.block_size)
    r.block_manager.allocate(s)
    s.num_new_tokens = len(s.token_ids) - s.num_cached_tokens
    pk = r._pack([s])
    ids, pos, ctx, _, _ = r._to_device(pk)
    with torch.inference_mode():
        l1 = r.model.forward(ids, pos, ctx, r.kv_layers, r.kv_scale_layers)[0].float().cpu()
    assert torch.nn.functional.cosine_similarity(lf, l1, dim=0).item() > 0.995
    for fused in ("fused", "fused_rs"):
        _check_greedy_margin(res[fused], res["nccl"], "out")
        _check_greedy_margin(res[fused], res["nccl"], "short")


def _check_greedy_margin(a, b, key):
    """Greedy outputs of two backends agree exactly, or first differ where the two chosen tokens
    are within the backends' logit noise.

    Both runs' sequences are scored by teacher forcing on both backends.  `noise` is the largest
    |logit difference| between the backends over identical contexts; at a sequence's first
    divergence (identical prefix), backend b's logits may separate the two chosen tokens by at
    most 2 noise + 1e-3: a larger margin would mean a wrong token, not a rounding tie.
    """
    seqs_a, seqs_b = a[key], b[key]
    scores_a, scores_b = a["scores"][key], b["scores"][key]
    firsts = [next((j for j, (u, v) in enumerate(zip(x, y)) if u != v), None) for x, y in zip(seqs_a, seqs_b)]
    # logits at position j depend on tokens 0..j only: positions before the first divergence
    # were computed on identical contexts by both backends
    noise = max((sa[:c] - sb[:c]).abs().max().item()
                for sa, sb, f, x in zip(scores_a, scores_b, firsts, seqs_a)
                for c in [len(x) if f is None else f] if c > 0)
    for i, (x, y) in enumerate(zip(seqs_a, seqs_b)):
        assert len(x) == len(y)
        first = firsts[i]
        if first is None:
            continue
        lb = scores_b[i][first - 1]  # logits that chose position `first` (same prefix in both runs)
        gap = abs(lb[x[first]].item() - lb[y[first]].item())
        assert gap <= 2 * noise + 1e-3, f"sequence {i}: tokens differ at {first} with margin {gap} > noise {noise}"


def _rs_worker(rank, world, port, out_path):
    """GEMM -> reduce-scatter -> residual + RMSNorm -> all-gather against an fp32 reference."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from nanovllm_self_b200.ops.cuda_ops import CudaOps
    from nanovllm_self_b200.parallel.state import init_tensor_parallel
    from nanovllm_self_b200.parallel.symm import SymmetricWorkspace
    tp = init_tensor_parallel(world, "cuda")
    dev = tp.device
    ops = CudaOps()
    H, K, eps = 1024, 512, 1e-6
    symm = SymmetricWorkspace(tp, rows=512, hidden=H, timeout_s=5.0)
    wn = (1 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(1))).to(torch.bfloat16).to(dev)
    errs = []
    for T in (1, 5, 64, 200, 256):
        g = torch.Generator().manual_seed(T)
        xs = [torch.randn(T, K, generator=g).to(torch.bfloat16) for _ in range(world)]
        ws = [(torch.randn(H, K, generator=g) * 0.05).to(torch.bfloat16) for _ in range(world)]
        rs = [torch.randn(T, H, generator=g).to(torch.bfloat16) for _ in range(world)]
        # residual stream: first an ordinary reduction (no residual) of the rs partials
        h0 = symm.input_buffer(T)
        h0.copy_(rs[rank].to(dev))
        symm.allreduce_add_rmsnorm(h0, None, wn, eps, ops)
        res = sum(r.float() for r in rs).to(torch.bfloat16).float()
        x = xs[rank].to(dev)
        w = ws[rank].to(dev)
        for call in range(2):  # twice: the call numbers advance, the buffers are reused
            symm.linear_rs(x, w, ops)
            out, _ = symm.rs_add_rmsnorm(T, wn, eps, ops)
            torch.cuda.synchronize()
            part = sum((xx.float() @ ww.float().t()).to(torch.bfloat16).float() for xx, ww in zip(xs, ws))
            v = (part + res).to(torch.bfloat16).float()
            ref = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + eps) * wn.float().cpu()
            e = (out.float().cpu() - ref).abs() / (ref.abs() + 1.0)
            errs.append((T, call, e.max().item()))
            # the owner's residual rows now hold v
            rr = symm.rs_rows(T)
            r0, r1 = rank * rr, min(T, (rank + 1) * rr)
            if r1 > r0:
                # relative like the output check: the GEMM's fp32 summation order differs from
                # torch's, so a bf16 partial (and hence v) may differ by one bf16 step
                rv = v[r0:r1]
                re = ((symm.RES[r0:r1].float().cpu() - rv).abs() / (rv.abs() + 1.0)).max().item()
                errs.append((T, call, re))
            res = v
    # the same pair of calls captured in a CUDA graph and replayed twice
    T = 64
    x = torch.randn(T, K, device=dev).to(torch.bfloat16)
    w = (torch.randn(H, K, device=dev) * 0.05).to(torch.bfloat16)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        symm.linear_rs(x, w, ops)  # tunes this shape outside the capture
        symm.rs_add_rmsnorm(T, wn, eps, ops)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    dist.barrier()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        symm.linear_rs(x, w, ops)
        symm.rs_add_rmsnorm(T, wn, eps, ops)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    del graph
    err = symm.error()
    gerr = ops.C.gemm_error(False)
    dist.barrier()
    if rank == 0:
        torch.save({"errs": errs, "err": err, "gemm_err": gerr}, out_path)
    symm.close()
    dist.destroy_process_group()


def _sample_worker(rank, world, port, out_path):
    """Vocab-parallel sampling in one kernel per step equals sampling the full logits on one GPU."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from nanovllm_self_b200.ops.cuda_ops import CudaOps
    from nanovllm_self_b200.parallel.state import init_tensor_parallel
    from nanovllm_self_b200.parallel.symm import SymmetricWorkspace
    tp = init_tensor_parallel(world, "cuda")
    dev = tp.device
    ops = CudaOps()
    # 48 rows, and more rows than CTAs that can be resident at once (each CTA then loops)
    cap = int(ops.C.sample_rows_capacity())
    big = cap + 20
    symm = SymmetricWorkspace(tp, rows=64, hidden=256, timeout_s=5.0, sample_rows=big)
    V = 151936
    per = (V + world - 1) // world
    res = {}
    for s, rows in enumerate((48, 48, 48, big)):
        g = torch.Generator().manual_seed(4 + s)
        logits = (torch.randn(rows, V, generator=g) * 3).to(dev)
        temps = torch.tensor([0.0, 1.0, 0.7, 1.3], device=dev).repeat((rows + 3) // 4)[:rows].contiguous()
        top_p = torch.tensor([1.0, 0.9, 0.5, 1.0], device=dev).repeat((rows + 3) // 4)[:rows].contiguous()
        step = torch.tensor([3, s], dtype=torch.int64, device=dev)
        shard = logits[:, rank * per:min(V, (rank + 1) * per)].contiguous()
        tok_tp = symm.sample_rows(shard, temps, top_p, step, rank * per, ops)
        tok_one = torch.empty(rows, dtype=torch.int32, device=dev)
        ops.C.sample_rows(logits, 0, temps, top_p, step, tok_one, None)
        torch.cuda.synchronize()
        res[s] = (tok_tp.cpu(), tok_one.cpu())
        del logits, shard
    err = ops.C.sample_error(False)
    dist.barrier()
    if rank == 0:
        torch.save({"res": res, "err": err}, out_path)
    symm.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_vocab_parallel_sampler_matches_one_gpu(tmp_path):
    out = tmp_path / "sample.pt"
    mp.spawn(_sample_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    res = torch.load(out)
    assert res["err"] == 0
    for s, (a, b) in res["res"].items():
        assert torch.equal(a, b), f"step {s}: {(a != b).sum().item()} rows differ"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_gemm_reduce_scatter_norm_allgather_matches_fp32(tmp_path):
    out = tmp_path / "rs.pt"
    mp.spawn(_rs_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    res = torch.load(out)
    assert res["err"] == 0 and res["gemm_err"] == 0
    for T, call, e in res["errs"]:
        assert e < 3e-2, f"T={T} call={call}: relative error {e}"


def _timeout_worker(rank, world, port, out_path):
    # A peer that never arrives: rank 1 skips one all-reduce (it decides so on the host and
    # waits there).  Rank 0's kernel must give up after its 1 s bound, record the error word
    # and return, leaving the context usable; nothing faults or hangs.
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import time
    import torch.distributed as dist
    from nanovllm_self_b200.ops.cuda_ops import CudaOps
    from nanovllm_self_b200.parallel.state import init_tensor_parallel
    from nanovllm_self_b200.parallel.symm import SymmetricWorkspace
    tp = init_tensor_parallel(world, "cuda")
    ops = CudaOps()
    symm = SymmetricWorkspace(tp, rows=64, hidden=256, timeout_s=1.0)
    w = torch.ones(256, device=tp.device, dtype=torch.bfloat16)
    h = symm.input_buffer(8)
    h.fill_(1.0)
    out, _ = symm.allreduce_add_rmsnorm(h, None, w, 1e-6, ops)  # both ranks: completes
    torch.cuda.synchronize()
    ok_first = symm.error() == 0 and bool(torch.isfinite(out.float()).all())
    dist.barrier()
    res = None
    if rank == 0:
        h = symm.input_buffer(8)
        h.fill_(1.0)
        t0 = time.time()
        symm.allreduce_add_rmsnorm(h, None, w, 1e-6, ops)  # rank 1 never joins this call
        torch.cuda.synchronize()
        res = {"elapsed_s": time.time() - t0, "err": symm.error(reset=True), "ok_first": ok_first}
        x = torch.ones(4, device=tp.device) * 3  # the context still runs work
        res["after"] = float(x.sum().item())
        torch.save(res, out_path)
    dist.barrier()
    symm.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_allreduce_peer_timeout_reports_error(tmp_path):
    out = tmp_path / "timeout.pt"
    mp.spawn(_timeout_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    res = torch.load(out)
    assert res["ok_first"]
    assert res["err"] == 110          # the entry barrier of the one-shot kernel gave up
    assert 0.8 < res["elapsed_s"] < 10.0
    assert res["after"] == 12.0
