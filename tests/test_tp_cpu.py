"""Tensor parallelism on CPU ranks (gloo): TP=2 greedy tokens equal TP=1.

Mirrors the reference's TP check (token equality across TP degrees,
``scripts/run_tp_memory_consistency_matrix.sh:45-60``), run as local processes over the
gloo backend instead of GPUs: sharded q/k/v/gate/up by rows, o/down by columns,
vocab-parallel embedding and lm_head, reductions via all_reduce.
"""
import json
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from nanovllm_self_b200 import LLM, SamplingParams


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _prompts():
    g = torch.Generator().manual_seed(3)
    return [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (9, 30, 17)]


def _kw():
    return dict(device="cpu", dtype="fp32", block_size=16, max_model_len=256, num_blocks=64, comm_backend="nccl")


def _worker(rank, world, port, out_path, temperature, model="tiny"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    llm = LLM(model, tensor_parallel_size=world, **_kw())
    out = llm.generate(_prompts(), SamplingParams(temperature=temperature, max_tokens=12, ignore_eos=True))
    with open(f"{out_path}.{rank}", "w") as f:
        json.dump(out, f)
    import torch.distributed as dist
    dist.barrier()
    # leave without tearing the gloo group down: its destructor can race with its own
    # threads at interpreter exit (std::terminate), which is a harness artefact, not a result
    os._exit(0)


@pytest.mark.parametrize("temperature", [0.0, 0.9])
def test_tp2_equals_tp1_on_cpu(tmp_path, temperature):
    ref = LLM("tiny", **_kw()).generate(_prompts(), SamplingParams(temperature=temperature, max_tokens=12,
                                                                    ignore_eos=True))
    out_path = str(tmp_path / "tp")
    mp.spawn(_worker, args=(2, _free_port(), out_path, temperature), nprocs=2, join=True)
    outs = [json.load(open(f"{out_path}.{r}")) for r in range(2)]
    assert outs[0] == outs[1], "ranks disagree"
    if temperature == 0.0:
        assert outs[0] == ref


@pytest.mark.parametrize("world", [4, 8])
def test_tp4_tp8_equal_tp1_on_cpu(tmp_path, world):
    """Qwen3-8B's 2:1 query / KV head ratio sharded 4 and 8 ways (at TP8 one KV head per rank, the
    layout of Qwen3-8B at TP8): greedy tokens equal the one-rank engine's."""
    sp = SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True)
    ref = LLM("tiny-tp8", **_kw()).generate(_prompts(), sp)
    out_path = str(tmp_path / "tp")
    mp.spawn(_worker, args=(world, _free_port(), out_path, 0.0, "tiny-tp8"), nprocs=world, join=True)
    outs = [json.load(open(f"{out_path}.{r}")) for r in range(world)]
    assert all(o == outs[0] for o in outs), "ranks disagree"
    assert outs[0] == ref
