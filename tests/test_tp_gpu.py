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


def _kw(backend):
    return dict(max_model_len=2048, max_num_seqs=16, num_blocks=64, cuda_graph_max_bs=16, comm_backend=backend)


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
    err = llm.comm.symm.error() if llm.comm.symm is not None else 0
    if rank == 0:
        torch.save({"out": out, "logits": logits, "err": err}, out_path)
    llm.shutdown()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_fused_matches_nccl_and_tp1(tmp_path):
    from nanovllm_self_b200 import LLM
    from nanovllm_self_b200.engine.sequence import Sequence
    from nanovllm_self_b200.sampling_params import SamplingParams
    res = {}
    for backend in ("fused", "nccl"):
        path = str(tmp_path / f"{backend}.pt")
        mp.spawn(_worker, args=(2, _free_port(), path, backend), nprocs=2, join=True)
        res[backend] = torch.load(path)
    assert res["fused"]["err"] == 0
    lf, ln = res["fused"]["logits"], res["nccl"]["logits"]
    assert torch.nn.functional.cosine_similarity(lf, ln, dim=0).item() > 0.999
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
    agree = sum(a == b for x, y in zip(res["fused"]["out"], res["nccl"]["out"]) for a, b in zip(x, y))
    total = sum(len(x) for x in res["fused"]["out"])
    assert agree / total > 0.9


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
