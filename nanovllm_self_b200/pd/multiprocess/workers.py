"""Persistent prefill and decode worker processes.

Reference: ``pd_self/multiprocess/persistent_prefill_worker.py`` and
``persistent_decode_worker.py``.  Same protocol shape: the driver drops
``<base>.request.json`` into a prefill worker's directory; the prefill worker runs the
prompt to its first token, writes ``<base>.payload.pkl`` into the target decode worker's
directory and moves the KV by the chosen backend; the decode worker restores it and
decodes, writing ``<base>.decode_metrics.json`` then ``<base>.decode_done``.  Errors go
to ``<base>.<stage>_error.json`` and the worker keeps serving; ``worker_state.json``
reports load for the router; a ``shutdown`` file stops the worker after it drains.

KV backends:

* ``shared_memory``: KV staged through POSIX shared memory (host copy);
* ``sync_gpu``: NCCL point-to-point send/recv in one NCCL world of P + D ranks; the
  decode side writes ``recv_ready`` before posting its receive (deadlock-free order);
* ``ipc_push`` (B200 path, no staging): the decode worker exports its KV pool through
  CUDA IPC once; for each handoff it allocates destination blocks and answers
  ``recv_ready`` with their ids; the prefill worker's push kernel copies its blocks
  straight into the decode pool over NVLink and signals ``push_done``.

Every wait on a peer is bounded (``--handshake-timeout-s``).

A worker can be a tensor-parallel group (``--tp N``, launched with ``torch.distributed.run``,
rank r on GPU ``--gpu-offset + r``): the group's rank 0 reads the work directory and decides,
and every decision (serve this request, admit this payload, run a decode step, stop) is
broadcast to the other ranks over a CPU control group, so all ranks run the same engine
operations in lockstep.  KV moves shard by shard: prefill rank r hands its KV heads to decode
rank r (``shared_memory``: one payload file per rank; ``ipc_push``: one exported pool per
decode rank, one ``push_done`` per prefill rank).  ``sync_gpu`` needs one NCCL world across
P and D and stays TP=1.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
import traceback
from pathlib import Path

import torch

from ...config import EngineConfig
from ...engine.model_runner import ModelRunner
from ...parallel.state import TPState
from ..decode_engine import DecodeEngine
from ..kv_connector import KVConnector
from ..kv_store import DictKVStoreBackend, SharedMemoryKVStoreBackend, SyncGpuKVStoreBackend
from ..prefill_engine import PrefillEngine
from .control_plane import WorkDir

BACKENDS = ("shared_memory", "sync_gpu", "ipc_push")


def add_common_args(ap: argparse.ArgumentParser) -> None:
    ap.add_argument("--work-dir", required=True)
    ap.add_argument("--model", default="tiny")
    ap.add_argument("--model-path", default=None)
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--dtype", default="bf16")
    ap.add_argument("--backend", choices=BACKENDS, default="shared_memory")
    ap.add_argument("--block-size", type=int, default=256)
    ap.add_argument("--num-blocks", type=int, default=-1)
    ap.add_argument("--max-num-seqs", type=int, default=64)
    ap.add_argument("--max-num-batched-tokens", type=int, default=16384)
    ap.add_argument("--max-model-len", type=int, default=4096)
    ap.add_argument("--kv-cache-quant-mode", default="none")
    ap.add_argument("--gpu-memory-utilization", type=float, default=0.85)
    ap.add_argument("--global-rank", type=int, default=0)
    ap.add_argument("--world-size", type=int, default=1)
    ap.add_argument("--nccl-port", type=int, default=29600)
    ap.add_argument("--poll-s", type=float, default=0.002)
    ap.add_argument("--handshake-timeout-s", type=float, default=120.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--enforce-eager", action="store_true")
    ap.add_argument("--tp", type=int, default=1, help="tensor-parallel size of this worker (torchrun launch)")
    ap.add_argument("--gpu-offset", type=int, default=0, help="rank r of the group uses GPU gpu_offset + r")
    ap.add_argument("--comm-backend", default="fused")
    # backpressure (reference persistent_prefill_worker.py:834-842, persistent_decode_worker.py:704-727)
    ap.add_argument("--max-pending-sends", type=int, default=0,
                    help="prefill: NCCL sends in flight before the worker completes them (0: no cap)")
    ap.add_argument("--max-active-decode-requests", type=int, default=0,
                    help="decode: requests admitted at once, restoring, pushed to or decoding (0: no cap)")
    ap.add_argument("--max-pending-recvs", type=int, default=0,
                    help="decode: NCCL receives in flight before new handoffs wait in the work directory (0: no cap)")


def build_runner(args, kv_pool_ipc: bool = False) -> ModelRunner:
    cfg = EngineConfig(kv_pool_ipc=kv_pool_ipc, model=None if args.model_path else args.model, model_path=args.model_path, device=args.device,
                       dtype=args.dtype, block_size=args.block_size, num_blocks=args.num_blocks,
                       max_num_seqs=args.max_num_seqs, max_num_batched_tokens=args.max_num_batched_tokens,
                       max_model_len=args.max_model_len, kv_cache_quant_mode=args.kv_cache_quant_mode,
                       gpu_memory_utilization=args.gpu_memory_utilization, seed=args.seed,
                       enforce_eager=args.enforce_eager, tensor_parallel_size=args.tp,
                       comm_backend=args.comm_backend)
    if args.tp > 1:
        from ...parallel.comm import TPComm
        from ...parallel.state import init_tensor_parallel
        kind = "cuda" if str(args.device).startswith("cuda") else "cpu"
        tp = init_tensor_parallel(args.tp, kind, timeout_s=args.handshake_timeout_s, gpu_offset=args.gpu_offset)
        cfg = cfg.replace(device=str(tp.device))
        comm = TPComm(tp, backend=cfg.comm_backend, config=cfg)
        return ModelRunner(cfg, tp, comm)
    dev = torch.device(args.device)
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    return ModelRunner(cfg, TPState(device=dev))


class GroupControl:
    """Lockstep control of a TP worker group: rank 0 decides, the other ranks follow.

    ``sync(cmd)`` returns rank 0's command on every rank (a pickled object broadcast over a
    CPU group); ``all_ok(flag)`` is True only if every rank passed True; ``barrier()`` waits
    for the whole group.  With one rank these are identities."""

    def __init__(self, tp: TPState):
        self.tp = tp
        self.group = None
        if tp.size > 1:
            import torch.distributed as dist
            self.group = dist.new_group(backend="gloo")

    @property
    def leader(self) -> bool:
        return self.tp.rank == 0

    def sync(self, cmd):
        if self.group is None:
            return cmd
        import torch.distributed as dist
        box = [cmd]
        dist.broadcast_object_list(box, src=0, group=self.group)
        return box[0]

    def all_ok(self, ok: bool) -> bool:
        if self.group is None:
            return ok
        import torch.distributed as dist
        t = torch.tensor([0 if ok else 1], dtype=torch.int32)
        dist.all_reduce(t, group=self.group)
        return int(t.item()) == 0

    def barrier(self) -> None:
        if self.group is not None:
            import torch.distributed as dist
            dist.barrier(group=self.group)


def rank_file(name: str, rank: int, size: int) -> str:
    """Per-rank artefact name: ``x.pkl`` -> ``x.rank2.pkl`` in a TP group, unchanged at TP=1."""
    if size == 1:
        return name
    stem, dot, ext = name.rpartition(".")
    return f"{stem}.rank{rank}.{ext}" if dot else f"{name}.rank{rank}"


def rank_name(name: str, tp: TPState) -> str:
    return rank_file(name, tp.rank, tp.size)


def init_world(args) -> None:
    if args.backend != "sync_gpu" or args.world_size <= 1:
        return
    import datetime
    import torch.distributed as dist
    kw = dict(backend="nccl" if str(args.device).startswith("cuda") else "gloo",
              init_method=f"tcp://127.0.0.1:{args.nccl_port}", rank=args.global_rank, world_size=args.world_size,
              timeout=datetime.timedelta(seconds=args.handshake_timeout_s))
    if str(args.device).startswith("cuda"):
        kw["device_id"] = torch.device(args.device)
    dist.init_process_group(**kw)


def _error(wd: WorkDir, base: str, stage: str, exc: BaseException) -> None:
    wd.write_json(f"{base}.{stage}_error.json", {"error": repr(exc), "traceback": traceback.format_exc(),
                                                 "time": time.time()})


# ======================================================================= prefill
class PrefillWorker:
    def __init__(self, args):
        self.args = args
        if args.tp > 1 and args.backend == "sync_gpu":
            raise ValueError("sync_gpu needs one NCCL world across P and D: use ipc_push or shared_memory with --tp")
        self.wd = WorkDir(args.work_dir)
        init_world(args)
        self.runner = build_runner(args)
        self.tp = self.runner.tp
        self.ctl = GroupControl(self.tp)
        cfg = self.runner.config
        if args.backend == "shared_memory":
            store = SharedMemoryKVStoreBackend()
        elif args.backend == "sync_gpu":
            store = SyncGpuKVStoreBackend(args.global_rank, peer_rank=None)
        else:
            store = DictKVStoreBackend()  # unused: ipc_push never stages
        self.store = store
        self.connector = KVConnector(cfg, "producer", f"prefill-{args.global_rank}-r{self.tp.rank}", store,
                                     export=args.backend != "ipc_push")
        self.connector.register_model_runner(self.runner)
        self.engine = PrefillEngine(cfg, None, self.runner, self.connector)
        self.pending_sends = []  # (state, base, decode WorkDir, metrics)
        self.peer_pools = {}     # decode work dir -> opened pool (ipc_push)
        self.seq_idx = 0
        self.processed = set()
        self.ctl.barrier()
        if self.ctl.leader:
            self.wd.write_json("worker_ready.json", {"pid": os.getpid(), "role": "prefill", "tp": self.tp.size,
                                                     "time": time.time()})

    def state(self, busy: bool) -> dict:
        queued = len([p for p in self.wd.glob("*.request.json") if p.name not in self.processed])
        return {"role": "prefill", "busy": busy, "queue_depth": queued, "pending_sends": len(self.pending_sends),
                "tp": self.tp.size, "time": time.time()}

    # ------------------------------------------------------------- ipc push
    def _peer_pool(self, dwd: WorkDir):
        key = str(dwd.path)
        if key not in self.peer_pools:
            name = rank_name("kv_pool.json", self.tp)  # this rank's counterpart in the decode group
            if not dwd.wait_for(name, self.args.handshake_timeout_s):
                raise TimeoutError(f"decode worker {key} never published its KV pool ({name})")
            info = dwd.read_json(name)
            from ...ops._ext import load
            C = load()
            raw = bytes.fromhex(info["handle"])
            ptr = C.symm_open(raw[:64])
            offset = int.from_bytes(raw[64:72], "little")
            flag_ptr, epoch = 0, 0
            if info.get("flag_offset"):
                # this worker's completion word in the decode pool's allocation; the sequence
                # continues from the word's current value (a restarted sender never reuses an
                # epoch the receiver already saw)
                slot = self.args.global_rank % int(C.PUSH_FLAG_SLOTS)
                flag_ptr = int(ptr) + int(info["flag_offset"]) + 4 * slot
                from ...parallel.symm import _DevPtr
                word = torch.as_tensor(_DevPtr(flag_ptr, 4), device=self.runner.device).view(torch.int32)
                epoch = int(word.cpu().item()) & 0xFFFFFFFF
                info = dict(info, slot=slot)
            self.peer_pools[key] = [ptr, info, offset, flag_ptr, epoch]
        return self.peer_pools[key]

    def _push(self, payload, dwd: WorkDir, base: str) -> None:
        meta = payload.transfer_meta
        if not dwd.wait_for(f"{base}.recv_ready", self.args.handshake_timeout_s):
            raise TimeoutError("decode worker did not answer recv_ready")
        dst = dwd.read_json(f"{base}.recv_ready")["dst_block_ids"]
        peer = self._peer_pool(dwd)
        ptr, info, offset, flag_ptr = peer[0], peer[1], peer[2], peer[3]
        if list(info["shape"][:2]) != list(self.runner.kv_cache.shape[:2]) or \
                list(info["shape"][3:]) != list(self.runner.kv_cache.shape[3:]) or info["dtype"] != str(self.runner.kv_cache.dtype):
            raise ValueError("decode KV pool layout differs from the prefill pool")
        from ...ops._ext import load
        C = load()
        r = self.runner
        src = torch.as_tensor(meta.src_block_table, dtype=torch.int32, device=r.device)
        dsti = torch.as_tensor(dst, dtype=torch.int32, device=r.device)
        C.kv_push(r.kv_cache, src, dsti, int(ptr) + offset, int(info["num_blocks"]))
        if r.kv_scale_cache is not None and r.config.kv_cache_quant_mode == "fp8":
            if not info.get("scale_offset"):
                raise ValueError("fp8 KV needs the decode pool's scales in the exported allocation")
            C.kv_push(r.kv_scale_cache, src, dsti, int(ptr) + int(info["scale_offset"]), int(info["num_blocks"]))
        done = {"time": time.time()}
        if flag_ptr:
            # device completion: the flag rises in stream order after the copies, and the decode
            # stream waits for it, so no host synchronisation sits between the push and decode
            # (later prefill kernels that reuse the source blocks run after the push in this stream)
            peer[4] = (peer[4] + 1) & 0xFFFFFFFF
            C.kv_push_signal(flag_ptr, peer[4])
            done.update(slot=info["slot"], epoch=peer[4])
        elif r.is_cuda:
            torch.cuda.synchronize(r.device)
        dwd.write_json(rank_name(f"{base}.push_done", self.tp), done)

    # ------------------------------------------------------------- requests
    def finalize_pending_sends(self, block: bool = False) -> None:
        keep = []
        for state, base, dwd, metrics in self.pending_sends:
            if block:
                self.store.wait_transfer(state)
            if block or self.store.transfer_done(state):
                metrics["send_complete_time"] = time.time()
                dwd.write_json(f"{base}.prefill_metrics.json", metrics)
                dwd.touch(f"{base}.prefill_done")
            else:
                keep.append((state, base, dwd, metrics))
        self.pending_sends = keep

    def process_request(self, base: str, req: dict) -> None:
        """Run on every rank of the group (the command came from rank 0)."""
        leader = self.ctl.leader
        dwd = WorkDir(req.get("decode_work_dir") or self.args.work_dir)
        t0 = time.time()
        payload, metrics, err = None, None, None
        try:
            if self.args.backend == "sync_gpu":
                self.store.set_peer_rank(int(req["dst_rank"]))
            seq = self.engine.add_request(req["prompt_ids"], self.seq_idx, float(req.get("temperature", 0.0)),
                                          int(req.get("max_tokens", 64)), bool(req.get("ignore_eos", True)),
                                          request_id=req.get("request_id", base), session_id=req.get("session_id"))
            self.seq_idx += 1
            payloads = []
            while not payloads:
                payloads = self.engine.step()
                if not self.engine.last_step_scheduled and not payloads:
                    raise RuntimeError(f"prefill stalled: {self.engine.scheduler.last_schedule_info.reason}")
            payload = payloads[0]
            t1 = time.time()
            metrics = {"request_id": payload.request_id, "prefill_time_s": t1 - t0, "first_token": payload.token_ids[-1],
                       "num_prompt_tokens": payload.num_prompt_tokens, "prefill_start_time": t0,
                       "prefix_cache_hit": payload.prefix_cache_hit, "prefix_cached_tokens": payload.prefix_cached_tokens,
                       "tp": self.tp.size}
            dwd.write_pickle(rank_name(f"{base}.payload.pkl", self.tp), payload)
            metrics["payload_write_time_s"] = time.time() - t1
        except Exception as e:
            err = e
        if not self.ctl.all_ok(err is None):
            if leader:
                _error(dwd, base, "prefill", err or RuntimeError("a peer rank of the prefill group failed"))
            return
        try:
            if payload.finished or self.args.backend == "shared_memory":
                if leader:
                    dwd.write_json(f"{base}.prefill_metrics.json", metrics)
                    dwd.touch(f"{base}.prefill_done")
            elif self.args.backend == "sync_gpu":
                dwd.touch(f"{base}.payload_ready")
                tw = time.time()
                if not dwd.wait_for(f"{base}.recv_ready", self.args.handshake_timeout_s):
                    self.store.delete(payload.transfer_meta.handoff_id)  # nothing was sent: drop the KV
                    raise TimeoutError("decode worker did not post its receive")
                metrics["transfer_wait_time_s"] = time.time() - tw
                ts = time.time()
                st = self.store.submit_send(payload.transfer_meta.handoff_id)
                metrics["send_submit_time_s"] = time.time() - ts
                self.pending_sends.append((st, base, dwd, metrics))
            else:
                if leader:
                    dwd.touch(f"{base}.payload_ready")  # every rank's payload file is written
                tw = time.time()
                self._push(payload, dwd, base)
                metrics["push_time_s"] = time.time() - tw
        except Exception as e:
            err = e
        if self.args.backend != "ipc_push" or payload.finished:
            if err is not None:
                _error(dwd, base, "prefill", err)
            return
        ok = self.ctl.all_ok(err is None)
        if leader:
            if ok:
                dwd.write_json(f"{base}.prefill_metrics.json", metrics)
                dwd.touch(f"{base}.prefill_done")
            else:
                _error(dwd, base, "prefill", err or RuntimeError("a peer rank of the prefill group failed to push"))

    def _next_command(self, idle_since: float, max_idle_s) -> dict:
        """Rank 0: what the group does next."""
        # at the send cap, complete the sends in flight before taking another request
        cap = getattr(self.args, "max_pending_sends", 0)
        self.finalize_pending_sends(block=cap > 0 and len(self.pending_sends) >= cap)
        for path in self.wd.glob("*.request.json"):
            if path.name in self.processed:
                continue
            base = path.name[:-len(".request.json")]
            self.processed.add(path.name)
            try:
                req = json.loads(path.read_text())
            except Exception as e:
                _error(self.wd, base, "prefill", e)
                path.unlink(missing_ok=True)
                continue
            path.unlink(missing_ok=True)
            self.wd.write_json("worker_state.json", self.state(True))
            return {"op": "prefill", "base": base, "req": req}
        self.wd.write_json("worker_state.json", self.state(False))
        if self.wd.shutdown_requested():
            return {"op": "stop"}
        if max_idle_s is not None and time.time() - idle_since > max_idle_s:
            return {"op": "stop"}
        return {"op": "idle"}

    def serve(self, max_idle_s: float | None = None) -> None:
        idle_since = time.time()
        while True:
            cmd = self.ctl.sync(self._next_command(idle_since, max_idle_s) if self.ctl.leader else None)
            if cmd["op"] == "prefill":
                self.process_request(cmd["base"], cmd["req"])
                idle_since = time.time()
            elif cmd["op"] == "stop":
                break
            else:
                time.sleep(self.args.poll_s)
        self.finalize_pending_sends(block=True)
        self.shutdown()

    def shutdown(self) -> None:
        from ...ops._ext import available, load
        if self.peer_pools and available():
            C = load()
            for entry in self.peer_pools.values():  # [ptr, info, offset, flag_ptr, epoch]
                try:
                    C.symm_close(int(entry[0]))
                except RuntimeError:
                    pass
            self.peer_pools.clear()
        self.runner.release_graphs()
        _close_worlds(self)


def _close_worlds(worker) -> None:
    import torch.distributed as dist
    if worker.tp.size > 1 and worker.runner.comm is not None:
        worker.runner.comm.close()
    if dist.is_initialized() and (worker.tp.size > 1 or (worker.args.backend == "sync_gpu" and worker.args.world_size > 1)):
        dist.destroy_process_group()


# ======================================================================== decode
class DecodeWorker:
    def __init__(self, args):
        self.args = args
        if args.tp > 1 and args.backend == "sync_gpu":
            raise ValueError("sync_gpu needs one NCCL world across P and D: use ipc_push or shared_memory with --tp")
        self.wd = WorkDir(args.work_dir)
        init_world(args)
        self.runner = build_runner(args, kv_pool_ipc=args.backend == "ipc_push")
        self.tp = self.runner.tp
        self.ctl = GroupControl(self.tp)
        cfg = self.runner.config
        if args.backend == "shared_memory":
            store = SharedMemoryKVStoreBackend()
        elif args.backend == "sync_gpu":
            store = SyncGpuKVStoreBackend(args.global_rank)
        else:
            store = DictKVStoreBackend()
        self.store = store
        self.connector = KVConnector(cfg, "consumer", f"decode-{args.global_rank}-r{self.tp.rank}", store)
        self.connector.register_model_runner(self.runner)
        self.engine = DecodeEngine(cfg, None, self.runner, self.connector)
        self.pending_recvs = {}   # base -> (state, payload)
        self.pending_push = {}    # base -> (payload, seq blocks, t0)
        self.push_status = {}     # base -> device status of the push completion wait
        self.active_bases = {}    # request_id -> (base, start time, restore_s)
        self.seen = set()
        if args.backend == "ipc_push":
            self._export_pool()
        self.ctl.barrier()
        if self.ctl.leader:
            self.wd.write_json("worker_ready.json", {"pid": os.getpid(), "role": "decode", "tp": self.tp.size,
                                                     "time": time.time()})

    def _export_pool(self) -> None:
        r = self.runner
        handle = r.export_kv_pool()
        self.wd.write_json(rank_name("kv_pool.json", self.tp), {
            "handle": handle.hex(), "num_blocks": r.num_blocks, "dtype": str(r.kv_cache.dtype),
            "shape": list(r.kv_cache.shape), "scale_offset": r.kv_scale_offset,
            "flag_offset": r.push_flag_offset})

    def state(self) -> dict:
        return {"role": "decode", "busy": bool(self.engine.scheduler.running), "active": len(self.engine.active),
                "pending_recvs": len(self.pending_recvs), "pending_push": len(self.pending_push),
                "tp": self.tp.size, "time": time.time()}

    def _finish(self, req) -> None:
        base, t_start, restore_s = self.active_bases.pop(req.request_id)
        status = self.push_status.pop(base, None)
        if status is not None:
            # every rank of the group finishes the same requests in the same order (lockstep
            # steps), so this agreement is a group collective like the step's own
            ok = self.ctl.all_ok(int(status.item()) == 1)
            if not ok:
                if self.ctl.leader:
                    _error(self.wd, base, "decode",
                           RuntimeError("the KV push never signalled completion (device wait timed out)"))
                return
        if not self.ctl.leader:
            return
        seq = req.seq
        self.wd.write_json(f"{base}.decode_metrics.json", {
            "request_id": req.request_id, "output_ids": seq.completion_token_ids,
            "decode_step_tokens": seq.completion_token_ids[1:], "restore_time_s": restore_s,
            "decode_time_s": req.decode_time_s, "decode_compute_time_s": sum(req.step_amortized_s),
            "num_decode_steps": len(req.step_wall_s), "finish_time": time.time(), "start_time": t_start})
        self.wd.touch(f"{base}.decode_done")

    def _admit(self, base: str) -> None:
        """Every rank: read this rank's payload and start receiving or restoring it."""
        payload = self.wd.read_pickle(rank_name(f"{base}.payload.pkl", self.tp))
        if payload.finished:
            if self.ctl.leader:
                self.wd.write_json(f"{base}.decode_metrics.json", {
                    "request_id": payload.request_id, "output_ids": payload.token_ids[payload.num_prompt_tokens:],
                    "decode_step_tokens": [], "finish_time": time.time()})
                self.wd.touch(f"{base}.decode_done")
            return
        t0 = time.time()
        if self.args.backend == "shared_memory":
            path = str(self.wd.f(rank_name(f"{base}.payload.pkl", self.tp)))
            req = self.engine.restore_active_payload(payload, path)
            self.active_bases[req.request_id] = (base, t0, time.time() - t0)
        elif self.args.backend == "sync_gpu":
            self.wd.touch(f"{base}.recv_ready")  # before posting the receive
            st = self.store.submit_recv_by_ref(
                payload.transfer_meta.storage_ref, self.runner.device,
                num_cached_tokens=payload.transfer_meta.num_cached_tokens,
                num_kv_blocks=payload.transfer_meta.num_kv_blocks,
                last_block_num_tokens=payload.transfer_meta.last_block_num_tokens,
                kv_cache_quant_mode=payload.transfer_meta.kv_cache_quant_mode)
            self.pending_recvs[base] = (st, payload, t0)
        else:
            n = payload.transfer_meta.num_kv_blocks
            blocks = self.runner.block_manager.allocate_block(n)  # identical on every rank
            if self.ctl.leader:
                self.wd.write_json(f"{base}.recv_ready", {"dst_block_ids": blocks})
            self.pending_push[base] = (payload, blocks, t0)

    def _restore_pushed(self, base: str) -> None:
        payload, blocks, t0 = self.pending_push.pop(base)
        done = self.wd.read_json(self._push_done_name(base, self.tp.rank))
        if "epoch" in done and self.runner.push_flags is not None:
            # the stream (and so every decode step of this request) waits for the device flag
            self.push_status[base] = self.runner.wait_push(int(done["slot"]), int(done["epoch"]),
                                                           self.args.handshake_timeout_s)
        seq = self.engine._new_sequence(payload)
        seq.block_table = blocks
        self.engine._restore_block_manager_meta(seq)
        self.engine.scheduler.running.append(seq)
        from ..decode_engine import ActiveDecodeRequest
        req = ActiveDecodeRequest(payload.request_id, seq, time.time() - t0)
        self.engine.active[payload.request_id] = req
        self.active_bases[req.request_id] = (base, t0, time.time() - t0)

    def _leader_ops(self, idle_since: float, max_idle_s) -> list:
        """Rank 0: the operations the group applies this iteration, in order."""
        ops = []
        marker = "prefill_done" if self.args.backend == "shared_memory" else "payload_ready"
        names = [p.name[:-len(f".{marker}")] for p in self.wd.glob(f"*.{marker}")]
        if marker != "prefill_done":
            # a request that finished on the prefill side arrives as prefill_done only
            names += [p.name[:-len(".prefill_done")] for p in self.wd.glob("*.prefill_done")
                      if self.wd.exists(p.name[:-len(".prefill_done")] + ".payload.pkl")
                      or self.wd.exists(p.name[:-len(".prefill_done")] + ".payload.rank0.pkl")]
        # admission caps: handoffs beyond them stay in the work directory until a slot frees up
        cap = getattr(self.args, "max_active_decode_requests", 0)
        recv_cap = getattr(self.args, "max_pending_recvs", 0)
        in_flight = len(self.engine.active) + len(self.pending_push) + len(self.pending_recvs)
        recvs = len(self.pending_recvs)
        for base in sorted(names):
            if base in self.seen:
                continue
            if (cap > 0 and in_flight >= cap) or (recv_cap > 0 and self.args.backend == "sync_gpu" and recvs >= recv_cap):
                break
            recvs += self.args.backend == "sync_gpu"
            self.seen.add(base)
            ops.append(("admit", base))
            in_flight += 1
        for base, (payload, blocks, t0) in self.pending_push.items():
            done = [self.wd.exists(self._push_done_name(base, r)) for r in range(self.tp.size)]
            if all(done):
                ops.append(("pushed", base))
            elif time.time() - t0 > self.args.handshake_timeout_s:
                ops.append(("push_timeout", base))
        for base, (st, payload, t0) in self.pending_recvs.items():
            if self.store.transfer_done(st):
                ops.append(("received", base))
        busy = bool(self.engine.scheduler.running) or any(o[0] in ("admit", "pushed", "received") for o in ops)
        if not busy and not ops:
            if self.wd.shutdown_requested() and not self.pending_recvs and not self.pending_push:
                ops.append(("stop",))
            elif max_idle_s is not None and time.time() - idle_since > max_idle_s:
                ops.append(("stop",))
        return ops

    def _push_done_name(self, base: str, rank: int) -> str:
        return rank_file(f"{base}.push_done", rank, self.tp.size)

    def _apply(self, op) -> bool:
        """Every rank applies one operation; returns False on stop."""
        kind, base = op[0], (op[1] if len(op) > 1 else None)
        if kind == "stop":
            return False
        if kind == "admit":
            err = None
            try:
                self._admit(base)
            except Exception as e:
                err = e
            if not self.ctl.all_ok(err is None):
                self._drop(base)
                if self.ctl.leader:
                    _error(self.wd, base, "decode", err or RuntimeError("a peer rank of the decode group failed"))
        elif kind == "pushed":
            self._restore_pushed(base)
        elif kind == "push_timeout":
            payload, blocks, _ = self.pending_push.pop(base)
            self.runner.block_manager.free_blocks(blocks)
            if self.ctl.leader:
                _error(self.wd, base, "decode", TimeoutError("prefill worker never pushed the KV"))
        elif kind == "received":
            st, payload, t0 = self.pending_recvs.pop(base)
            item = self.store.finish_recv(st)
            req = self.engine.restore_active_payload_from_kv_item(payload, item)
            self.active_bases[req.request_id] = (base, t0, time.time() - t0)
        return True

    def _drop(self, base: str) -> None:
        """Undo a partial admission on this rank (another rank failed)."""
        if base in self.pending_push:
            _, blocks, _ = self.pending_push.pop(base)
            self.runner.block_manager.free_blocks(blocks)
        for rid, (b, _, _) in list(self.active_bases.items()):
            if b == base:
                self.engine.abort_by_request_id(rid)
                self.active_bases.pop(rid, None)

    def _decode_step(self) -> None:
        err = None
        try:
            self.engine.continuous_step()
        except Exception as e:
            err = e
        if not self.ctl.all_ok(err is None):
            for rid, (base, _, _) in list(self.active_bases.items()):
                if self.ctl.leader:
                    _error(self.wd, base, "decode", err or RuntimeError("a peer rank of the decode group failed"))
                self.engine.abort_by_request_id(rid)
                self.active_bases.pop(rid, None)
                self.push_status.pop(base, None)
        for req in list(self.engine.finished_active):
            self._finish(req)
        self.engine.finished_active.clear()

    def serve(self, max_idle_s: float | None = None) -> None:
        idle_since = time.time()
        running = True
        while running:
            ops = self.ctl.sync(self._leader_ops(idle_since, max_idle_s) if self.ctl.leader else None)
            for op in ops:
                if not self._apply(op):
                    running = False
                    break
            if not running:
                break
            if self.engine.scheduler.running:  # identical on every rank
                self._decode_step()
                idle_since = time.time()
            elif not ops:
                time.sleep(self.args.poll_s)
            if self.ctl.leader:
                self.wd.write_json("worker_state.json", self.state())
        self.runner.release_graphs()
        _close_worlds(self)


def main(role: str, argv=None) -> None:
    ap = argparse.ArgumentParser(description=f"persistent {role} worker")
    add_common_args(ap)
    ap.add_argument("--max-idle-s", type=float, default=None)
    args = ap.parse_args(argv)
    w = PrefillWorker(args) if role == "prefill" else DecodeWorker(args)
    w.serve(max_idle_s=args.max_idle_s)


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2:])
