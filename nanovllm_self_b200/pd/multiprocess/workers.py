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


def build_runner(args, kv_pool_ipc: bool = False) -> ModelRunner:
    cfg = EngineConfig(kv_pool_ipc=kv_pool_ipc, model=None if args.model_path else args.model, model_path=args.model_path, device=args.device,
                       dtype=args.dtype, block_size=args.block_size, num_blocks=args.num_blocks,
                       max_num_seqs=args.max_num_seqs, max_num_batched_tokens=args.max_num_batched_tokens,
                       max_model_len=args.max_model_len, kv_cache_quant_mode=args.kv_cache_quant_mode,
                       gpu_memory_utilization=args.gpu_memory_utilization, seed=args.seed,
                       enforce_eager=args.enforce_eager)
    dev = torch.device(args.device)
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    return ModelRunner(cfg, TPState(device=dev))


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
        self.wd = WorkDir(args.work_dir)
        init_world(args)
        self.runner = build_runner(args)
        cfg = self.runner.config
        if args.backend == "shared_memory":
            store = SharedMemoryKVStoreBackend()
        elif args.backend == "sync_gpu":
            store = SyncGpuKVStoreBackend(args.global_rank, peer_rank=None)
        else:
            store = DictKVStoreBackend()  # unused: ipc_push never stages
        self.store = store
        self.connector = KVConnector(cfg, "producer", f"prefill-{args.global_rank}", store,
                                     export=args.backend != "ipc_push")
        self.connector.register_model_runner(self.runner)
        self.engine = PrefillEngine(cfg, None, self.runner, self.connector)
        self.pending_sends = []  # (state, base, decode WorkDir, metrics)
        self.peer_pools = {}     # decode work dir -> opened pool (ipc_push)
        self.seq_idx = 0
        self.processed = set()
        self.wd.write_json("worker_ready.json", {"pid": os.getpid(), "role": "prefill", "time": time.time()})

    def state(self, busy: bool) -> dict:
        queued = len([p for p in self.wd.glob("*.request.json") if p.name not in self.processed])
        return {"role": "prefill", "busy": busy, "queue_depth": queued, "pending_sends": len(self.pending_sends),
                "time": time.time()}

    # ------------------------------------------------------------- ipc push
    def _peer_pool(self, dwd: WorkDir):
        key = str(dwd.path)
        if key not in self.peer_pools:
            if not dwd.wait_for("kv_pool.json", self.args.handshake_timeout_s):
                raise TimeoutError(f"decode worker {key} never published its KV pool")
            info = dwd.read_json("kv_pool.json")
            from ...ops._ext import load
            C = load()
            raw = bytes.fromhex(info["handle"])
            ptr = C.symm_open(raw[:64])
            self.peer_pools[key] = (ptr, info, int.from_bytes(raw[64:72], "little"))
        return self.peer_pools[key]

    def _push(self, payload, dwd: WorkDir, base: str) -> None:
        meta = payload.transfer_meta
        if not dwd.wait_for(f"{base}.recv_ready", self.args.handshake_timeout_s):
            raise TimeoutError("decode worker did not answer recv_ready")
        dst = dwd.read_json(f"{base}.recv_ready")["dst_block_ids"]
        ptr, info, offset = self._peer_pool(dwd)
        if list(info["shape"][:2]) != list(self.runner.kv_cache.shape[:2]) or \
                list(info["shape"][3:]) != list(self.runner.kv_cache.shape[3:]) or info["dtype"] != str(self.runner.kv_cache.dtype):
            raise ValueError("decode KV pool layout differs from the prefill pool")
        from ...ops._ext import load
        C = load()
        r = self.runner
        src = torch.as_tensor(meta.src_block_table, dtype=torch.int32, device=r.device)
        dsti = torch.as_tensor(dst, dtype=torch.int32, device=r.device)
        C.kv_push(r.kv_cache, src, dsti, int(ptr) + offset, int(info["num_blocks"]))
        torch.cuda.synchronize(r.device)
        dwd.write_json(f"{base}.push_done", {"time": time.time()})

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

    def process_request(self, path: Path) -> None:
        base = path.name[:-len(".request.json")]
        req = json.loads(path.read_text())
        dwd = WorkDir(req.get("decode_work_dir") or self.args.work_dir)
        t0 = time.time()
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
                       "prefix_cache_hit": payload.prefix_cache_hit, "prefix_cached_tokens": payload.prefix_cached_tokens}
            dwd.write_pickle(f"{base}.payload.pkl", payload)
            metrics["payload_write_time_s"] = time.time() - t1
            if payload.finished or self.args.backend == "shared_memory":
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
                dwd.touch(f"{base}.payload_ready")
                tw = time.time()
                self._push(payload, dwd, base)
                metrics["push_time_s"] = time.time() - tw
                dwd.write_json(f"{base}.prefill_metrics.json", metrics)
                dwd.touch(f"{base}.prefill_done")
        except Exception as e:  # keep serving
            _error(dwd, base, "prefill", e)
        finally:
            self.processed.add(path.name)
            path.unlink(missing_ok=True)

    def serve(self, max_idle_s: float | None = None) -> None:
        idle_since = time.time()
        while True:
            self.finalize_pending_sends()
            reqs = [p for p in self.wd.glob("*.request.json") if p.name not in self.processed]
            if reqs:
                self.wd.write_json("worker_state.json", self.state(True))
                self.process_request(reqs[0])
                idle_since = time.time()
                continue
            self.wd.write_json("worker_state.json", self.state(False))
            if self.wd.shutdown_requested():
                break
            if max_idle_s is not None and time.time() - idle_since > max_idle_s:
                break
            time.sleep(self.args.poll_s)
        self.finalize_pending_sends(block=True)
        self.shutdown()

    def shutdown(self) -> None:
        from ...ops._ext import available, load
        if self.peer_pools and available():
            C = load()
            for ptr, _, _ in self.peer_pools.values():
                try:
                    C.symm_close(int(ptr))
                except RuntimeError:
                    pass
        self.runner.release_graphs()
        if self.args.backend == "sync_gpu" and self.args.world_size > 1:
            import torch.distributed as dist
            if dist.is_initialized():
                dist.destroy_process_group()


# ======================================================================== decode
class DecodeWorker:
    def __init__(self, args):
        self.args = args
        self.wd = WorkDir(args.work_dir)
        init_world(args)
        self.runner = build_runner(args, kv_pool_ipc=args.backend == "ipc_push")
        cfg = self.runner.config
        if args.backend == "shared_memory":
            store = SharedMemoryKVStoreBackend()
        elif args.backend == "sync_gpu":
            store = SyncGpuKVStoreBackend(args.global_rank)
        else:
            store = DictKVStoreBackend()
        self.store = store
        self.connector = KVConnector(cfg, "consumer", f"decode-{args.global_rank}", store)
        self.connector.register_model_runner(self.runner)
        self.engine = DecodeEngine(cfg, None, self.runner, self.connector)
        self.pending_recvs = {}   # base -> (state, payload)
        self.pending_push = {}    # base -> (payload, seq blocks)
        self.active_bases = {}    # request_id -> (base, start time, restore_s)
        self.seen = set()
        if args.backend == "ipc_push":
            self._export_pool()
        self.wd.write_json("worker_ready.json", {"pid": os.getpid(), "role": "decode", "time": time.time()})

    def _export_pool(self) -> None:
        r = self.runner
        handle = r.export_kv_pool()
        self.wd.write_json("kv_pool.json", {"handle": handle.hex(), "num_blocks": r.num_blocks,
                                            "dtype": str(r.kv_cache.dtype), "shape": list(r.kv_cache.shape)})

    def state(self) -> dict:
        return {"role": "decode", "busy": bool(self.engine.scheduler.running), "active": len(self.engine.active),
                "pending_recvs": len(self.pending_recvs), "pending_push": len(self.pending_push),
                "time": time.time()}

    def _finish(self, req) -> None:
        base, t_start, restore_s = self.active_bases.pop(req.request_id)
        seq = req.seq
        self.wd.write_json(f"{base}.decode_metrics.json", {
            "request_id": req.request_id, "output_ids": seq.completion_token_ids,
            "decode_step_tokens": seq.completion_token_ids[1:], "restore_time_s": restore_s,
            "decode_time_s": req.decode_time_s, "decode_compute_time_s": sum(req.step_amortized_s),
            "num_decode_steps": len(req.step_wall_s), "finish_time": time.time(), "start_time": t_start})
        self.wd.touch(f"{base}.decode_done")

    def _admit(self, base: str) -> None:
        payload = self.wd.read_pickle(f"{base}.payload.pkl")
        if payload.finished:
            self.wd.write_json(f"{base}.decode_metrics.json", {"request_id": payload.request_id,
                                                               "output_ids": payload.token_ids[payload.num_prompt_tokens:],
                                                               "decode_step_tokens": [], "finish_time": time.time()})
            self.wd.touch(f"{base}.decode_done")
            return
        t0 = time.time()
        if self.args.backend == "shared_memory":
            req = self.engine.restore_active_payload(payload, str(self.wd.f(f"{base}.payload.pkl")))
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
            blocks = self.runner.block_manager.allocate_block(n)
            self.wd.write_json(f"{base}.recv_ready", {"dst_block_ids": blocks})
            self.pending_push[base] = (payload, blocks, t0)

    def _poll_transfers(self) -> None:
        for base, (st, payload, t0) in list(self.pending_recvs.items()):
            if self.store.transfer_done(st):
                item = self.store.finish_recv(st)
                req = self.engine.restore_active_payload_from_kv_item(payload, item)
                self.active_bases[req.request_id] = (base, t0, time.time() - t0)
                del self.pending_recvs[base]
        for base, (payload, blocks, t0) in list(self.pending_push.items()):
            if self.wd.exists(f"{base}.push_done"):
                seq = self.engine._new_sequence(payload)
                seq.block_table = blocks
                self.engine._restore_block_manager_meta(seq)
                self.engine.scheduler.running.append(seq)
                from ..decode_engine import ActiveDecodeRequest
                req = ActiveDecodeRequest(payload.request_id, seq, time.time() - t0)
                self.engine.active[payload.request_id] = req
                self.active_bases[req.request_id] = (base, t0, time.time() - t0)
                del self.pending_push[base]
            elif time.time() - t0 > self.args.handshake_timeout_s:
                self.runner.block_manager.free_blocks(blocks)
                del self.pending_push[base]
                _error(self.wd, base, "decode", TimeoutError("prefill worker never pushed the KV"))

    def serve(self, max_idle_s: float | None = None) -> None:
        idle_since = time.time()
        marker = "prefill_done" if self.args.backend == "shared_memory" else "payload_ready"
        while True:
            for p in self.wd.glob(f"*.{marker}"):
                base = p.name[:-len(f".{marker}")]
                if base in self.seen:
                    continue
                self.seen.add(base)
                try:
                    self._admit(base)
                except Exception as e:
                    _error(self.wd, base, "decode", e)
            # a request that finished on the prefill side arrives as prefill_done only
            if marker != "prefill_done":
                for p in self.wd.glob("*.prefill_done"):
                    base = p.name[:-len(".prefill_done")]
                    if base not in self.seen and self.wd.exists(f"{base}.payload.pkl"):
                        self.seen.add(base)
                        try:
                            self._admit(base)
                        except Exception as e:
                            _error(self.wd, base, "decode", e)
            self._poll_transfers()
            if self.engine.scheduler.running:
                try:
                    self.engine.continuous_step()
                except Exception as e:
                    for rid, (base, _, _) in list(self.active_bases.items()):
                        _error(self.wd, base, "decode", e)
                        self.engine.abort_by_request_id(rid)
                        self.active_bases.pop(rid, None)
                for req in list(self.engine.finished_active):
                    self._finish(req)
                self.engine.finished_active.clear()
                idle_since = time.time()
            else:
                if self.wd.shutdown_requested() and not self.pending_recvs and not self.pending_push:
                    break
                if max_idle_s is not None and time.time() - idle_since > max_idle_s:
                    break
                time.sleep(self.args.poll_s)
            self.wd.write_json("worker_state.json", self.state())
        self.runner.release_graphs()
        if self.args.backend == "sync_gpu" and self.args.world_size > 1:
            import torch.distributed as dist
            if dist.is_initialized():
                dist.destroy_process_group()


def main(role: str, argv=None) -> None:
    ap = argparse.ArgumentParser(description=f"persistent {role} worker")
    add_common_args(ap)
    ap.add_argument("--max-idle-s", type=float, default=None)
    args = ap.parse_args(argv)
    w = PrefillWorker(args) if role == "prefill" else DecodeWorker(args)
    w.serve(max_idle_s=args.max_idle_s)


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2:])
