"""KV handoff bandwidth between two GPUs: the NVLink push kernel against NCCL point-to-point.

Run with two ranks (rank 0 prefill side, rank 1 decode side)::

    NCCL_NVLS_ENABLE=0 python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 \
        --master-addr 127.0.0.1 --master-port 29581 -m nanovllm_self_b200.benchmarks.push

Pools have the engine's layout [2, layers, blocks, kv_heads, block_size, head_dim] (Qwen3-8B:
36 layers, 8 KV heads, head dim 128; block 256 tokens, so one block is 36 MiB over all layers).
For n blocks (scattered ids on both sides) three ways to move them are timed:

* ``push``: the decode rank's pool is a CUDA IPC allocation; the prefill rank's push kernel copies the
  blocks straight into it over NVLink and raises the completion flag (one launch + one signal);
* ``nccl_p2p``: the reference's data path (``pd_self/kv_store.py:432-500``): gather the blocks into a
  contiguous tensor, send / recv it, scatter it into the decode pool;
* ``nccl_raw``: send / recv of one contiguous buffer of the same size (the link alone).

Each number is CUDA-event time per transfer over ``--iters`` transfers after warm-up (for ``push``
the sender's stream; for NCCL the max over the two ranks); one JSON line per n.
GiB/s = bytes moved / time.
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from ..ops._ext import load
from ..parallel.symm import _DevPtr


def _timed(fn, iters: int) -> float:
    """ms per call of fn() on this rank's stream, after two warm-up calls and a barrier."""
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def _max(v: float, dev) -> float:
    t = torch.tensor([v], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--block-size", type=int, default=256)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--num-blocks", type=int, default=80)
    ap.add_argument("--sizes", default="1,4,8,32")
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args(argv)
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    assert world == 2, "two ranks: 0 pushes, 1 receives"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", device_id=dev)
    C = load()
    shape = (2, args.layers, args.num_blocks, args.kv_heads, args.block_size, args.head_dim)
    nbytes = 2
    for s in shape:
        nbytes *= s
    flag_off = (nbytes + 255) // 256 * 256
    total = flag_off + 4 * int(C.PUSH_FLAG_SLOTS)
    ptr, handle = C.symm_alloc(total)
    raw = torch.as_tensor(_DevPtr(ptr, total), device=dev)
    pool = raw[:nbytes].view(torch.bfloat16).view(shape)
    flags = raw[flag_off:total].view(torch.int32)
    flags.zero_()
    pool.normal_()
    handles = [None, None]
    dist.all_gather_object(handles, handle)
    peer = C.symm_open(handles[1]) if rank == 0 else 0
    peer_flag = peer + flag_off if rank == 0 else 0
    block_bytes = nbytes // args.num_blocks
    epoch = [0]
    g = torch.Generator().manual_seed(0)
    for n in [int(x) for x in args.sizes.split(",")]:
        src_ids = torch.randperm(args.num_blocks, generator=g)[:n].to(torch.int32).to(dev)
        dst_ids = torch.randperm(args.num_blocks, generator=g)[:n].to(torch.int32).to(dev)
        moved = n * block_bytes
        res = {"n_blocks": n, "bytes": moved}

        def push_once():
            # rank 1's stream waits for the flag (another GPU raises it: never a same-GPU wait)
            epoch[0] += 1
            if rank == 0:
                C.kv_push(pool, src_ids, dst_ids, int(peer), args.num_blocks)
                C.kv_push_signal(int(peer_flag), epoch[0])
            else:
                C.kv_push_wait(int(flags[0].data_ptr()), epoch[0], int(10e9))
        ms = _timed(push_once, args.iters)
        t = _max(ms if rank == 0 else 0.0, dev)  # the sender's stream: copy + signal
        res["push_ms"] = round(t, 4)
        res["push_gib_s"] = round(moved / (t / 1e3) / 2 ** 30, 2)

        staging = torch.empty((2, args.layers, n) + shape[3:], dtype=torch.bfloat16, device=dev)

        def nccl_once():
            if rank == 0:
                torch.index_select(pool, 2, src_ids.long(), out=staging)
                dist.send(staging, dst=1)
            else:
                dist.recv(staging, src=0)
                pool.index_copy_(2, dst_ids.long(), staging)
        t = _max(_timed(nccl_once, args.iters), dev)
        res["nccl_p2p_ms"] = round(t, 4)
        res["nccl_p2p_gib_s"] = round(moved / (t / 1e3) / 2 ** 30, 2)

        def raw_once():
            if rank == 0:
                dist.send(staging, dst=1)
            else:
                dist.recv(staging, src=0)
        t = _max(_timed(raw_once, args.iters), dev)
        res["nccl_raw_ms"] = round(t, 4)
        res["nccl_raw_gib_s"] = round(moved / (t / 1e3) / 2 ** 30, 2)
        res["push_error"] = int(C.push_error(False))
        res["comm_error"] = int(C.comm_error(False))
        del staging
        dist.barrier()
        if rank == 0:
            print(json.dumps(res), flush=True)
    dist.barrier()
    if rank == 0:
        C.symm_close(int(peer))
    dist.barrier()
    C.symm_free(int(ptr))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
