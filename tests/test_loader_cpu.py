"""Checkpoint round trip on CPU: the seeded random weights written as a sharded HF safetensors
directory load back bit for bit, and two tensor-parallel ranks (gloo) slicing the same files
generate the one-rank engine's greedy tokens."""
import json
import os
import socket

import torch
import torch.multiprocessing as mp

from nanovllm_self_b200 import LLM, SamplingParams
from nanovllm_self_b200.models.configs import PRESETS
from nanovllm_self_b200.models.loader import has_checkpoint, hf_tensor_shapes, save_hf_checkpoint

KW = dict(device="cpu", dtype="fp32", block_size=16, max_model_len=256, num_blocks=32, comm_backend="nccl")
PROMPTS = [[3, 14, 15, 92, 65, 35, 89, 79], list(range(100, 131))]
SP = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)


def _write(tmp_path):
    path = str(tmp_path / "ckpt")
    save_hf_checkpoint(PRESETS["tiny"], path, seed=0, dtype=torch.float32, max_shard_bytes=1 << 20)
    return path


def test_sharded_checkpoint_loads_bit_for_bit(tmp_path):
    path = _write(tmp_path)
    assert has_checkpoint(path) and not has_checkpoint(str(tmp_path / "missing"))
    index = json.load(open(os.path.join(path, "model.safetensors.index.json")))["weight_map"]
    assert set(index) == set(hf_tensor_shapes(PRESETS["tiny"])) and len(set(index.values())) > 1
    a = LLM("tiny", **KW).model_runner.model       # seeded random init
    b = LLM(path, **KW).model_runner.model         # the same weights through the safetensors loader
    for la, lb in zip(a.layers, b.layers):
        for k, t in la.tensors().items():
            assert torch.equal(t, lb.tensors()[k]), k
    assert torch.equal(a.embed, b.embed) and torch.equal(a.lm_head, b.lm_head) and torch.equal(a.norm, b.norm)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, path, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    llm = LLM(path, tensor_parallel_size=2, **KW)
    res = llm.generate(PROMPTS, SP)
    with open(f"{out}.{rank}", "w") as f:
        json.dump(res, f)
    import torch.distributed as dist
    dist.barrier()
    os._exit(0)  # no gloo teardown at interpreter exit


def test_tp2_ranks_slice_the_checkpoint(tmp_path):
    path = _write(tmp_path)
    want = LLM(path, **KW).generate(PROMPTS, SP)
    out = str(tmp_path / "tok")
    mp.spawn(_rank, args=(_free_port(), path, out), nprocs=2, join=True)
    assert json.load(open(f"{out}.0")) == json.load(open(f"{out}.1")) == want
