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
