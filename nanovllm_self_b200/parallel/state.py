"""Tensor-parallel process state.

One process per GPU, launched by ``torchrun`` (``RANK``/``LOCAL_RANK``/``WORLD_SIZE``
from the environment), as in the reference's ``init_tensor_parallel``
(``nanovllm/distributed/parallel_state.py:12-51``).  Unlike the reference there is no
module global that the model reads at import time; :class:`TPState` is created once
per engine and passed to the model and comm layers.

``backend`` is ``"nccl"`` on GPUs and ``"gloo"`` for CPU multi-rank tests.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class TPState:
    rank: int = 0
    size: int = 1
    local_rank: int = 0
    group: object = None
    device: torch.device = torch.device("cpu")

    @property
    def is_first(self) -> bool:
        return self.rank == 0


_STATE = TPState()


def init_tensor_parallel(tp_size: int, device: str = "cuda", timeout_s: float = 600.0, gpu_offset: int = 0) -> TPState:
    """Initialise (or reuse) the default process group for ``tp_size`` ranks.

    Rank ``r`` uses GPU ``gpu_offset + LOCAL_RANK``, so two TP groups can share a node
    (for example a prefill group on GPUs 0-3 and a decode group on GPUs 4-7)."""
    global _STATE
    is_cuda = str(device).startswith("cuda")
    if tp_size == 1:
        if is_cuda:
            idx = torch.device(device).index
            if idx is None:
                idx = int(os.environ.get("LOCAL_RANK", 0)) if dist.is_initialized() else torch.cuda.current_device()
            torch.cuda.set_device(idx)
            dev = torch.device("cuda", idx)
        else:
            dev = torch.device("cpu")
        _STATE = TPState(rank=0, size=1, local_rank=0, group=None, device=dev)
        return _STATE
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != tp_size:
        raise ValueError(f"WORLD_SIZE={world} but tensor_parallel_size={tp_size}; launch with torchrun")
    rank = int(os.environ["RANK"])
    local_rank = int(os.environ.get("LOCAL_RANK", rank))
    if is_cuda:
        torch.cuda.set_device(gpu_offset + local_rank)
        dev = torch.device("cuda", gpu_offset + local_rank)
    else:
        dev = torch.device("cpu")
    if not dist.is_initialized():
        kw = dict(backend="nccl" if is_cuda else "gloo", rank=rank, world_size=world,
                  timeout=datetime.timedelta(seconds=timeout_s))
        if is_cuda:
            kw["device_id"] = dev
        dist.init_process_group(**kw)
    _STATE = TPState(rank=rank, size=tp_size, local_rank=local_rank, group=dist.group.WORLD, device=dev)
    return _STATE


def get_tp_state() -> TPState:
    return _STATE


def get_tp_rank() -> int:
    return _STATE.rank


def get_tp_size() -> int:
    return _STATE.size


def tp_all_reduce(x: torch.Tensor, state: TPState | None = None) -> torch.Tensor:
    """In-place SUM all-reduce over the TP group (the reference's NCCL path)."""
    st = state or _STATE
    if st.size == 1:
        return x
    dist.all_reduce(x, op=dist.ReduceOp.SUM, group=st.group)
    return x
