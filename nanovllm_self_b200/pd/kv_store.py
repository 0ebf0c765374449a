"""KV store backends for the prefill -> decode handoff.

Same backend family and method names as the reference (``pd_self/kv_store.py:93-651``):

* :class:`DictKVStoreBackend`: in-process dict (prefill and decode runners in one process);
* :class:`SharedMemoryKVStoreBackend`: POSIX shared memory for cross-process handoff.  The
  tensor's raw bytes are stored as-is (bf16 stays 2 bytes, fp8 1 byte); the reference
  up-casts bf16 to fp32 through numpy (:183-220), doubling the bytes moved;
* :class:`SyncGpuKVStoreBackend`: GPU-to-GPU over NCCL point-to-point, synchronous
  (``send_pending`` / ``pop_by_ref``) or asynchronous (``submit_send`` /
  ``submit_recv_by_ref`` / ``transfer_done`` / ``wait_transfer`` / ``finish_recv``), with
  per-request ``set_peer_rank`` for pool routing.

An item holds the KV blocks ``[2, L, n, kv_heads, block_size, head_dim]`` of one request
plus, for quantised caches, their scales.
"""
from __future__ import annotations

import threading
import uuid
from abc import ABC, abstractmethod
from dataclasses import dataclass, field
from multiprocessing import shared_memory
from typing import Optional

import numpy as np
import torch

from .payload import SharedMemoryKVRef, SyncGpuKVRef

_DTYPES = {
    "torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16, "torch.float32": torch.float32,
    "torch.int8": torch.int8, "torch.float8_e4m3fn": torch.float8_e4m3fn, "torch.uint8": torch.uint8,
}
# numpy carrier dtype with the same element size
_CARRIER = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}


def dtype_from_str(s: str) -> torch.dtype:
    if s not in _DTYPES:
        raise ValueError(f"unsupported dtype string {s}")
    return _DTYPES[s]


@dataclass
class KVStoreItem:
    kv_blocks: Optional[torch.Tensor]
    scale_blocks: Optional[torch.Tensor]
    num_cached_tokens: int
    num_kv_blocks: int
    last_block_num_tokens: int
    kv_cache_quant_mode: str = "none"
    storage_ref: object = None
    scale_storage_ref: object = None


@dataclass
class AsyncSendState:
    handoff_id: str
    works: list
    tensors: list = field(default_factory=list)  # keep alive until completion


@dataclass
class AsyncRecvState:
    handoff_id: str
    works: list
    kv: torch.Tensor
    scale: Optional[torch.Tensor]
    item: KVStoreItem


class KVStoreBackend(ABC):
    device_direct = False

    @abstractmethod
    def put(self, handoff_id: str, item: KVStoreItem) -> KVStoreItem: ...

    @abstractmethod
    def get(self, handoff_id: str) -> KVStoreItem: ...

    @abstractmethod
    def pop(self, handoff_id: str) -> KVStoreItem: ...

    @abstractmethod
    def delete(self, handoff_id: str) -> None: ...

    def delete_by_ref(self, ref) -> None:
        self.delete(getattr(ref, "handoff_id", ref))

    @abstractmethod
    def exists(self, handoff_id: str) -> bool: ...


class DictKVStoreBackend(KVStoreBackend):
    def __init__(self):
        self.store: dict[str, KVStoreItem] = {}
        self._lock = threading.Lock()

    def put(self, handoff_id, item):
        with self._lock:
            self.store[handoff_id] = item
        return item

    def get(self, handoff_id):
        with self._lock:
            if handoff_id not in self.store:
                raise KeyError(f"handoff {handoff_id} not found")
            return self.store[handoff_id]

    def pop(self, handoff_id):
        with self._lock:
            if handoff_id not in self.store:
                raise KeyError(f"handoff {handoff_id} not found")
            return self.store.pop(handoff_id)

    def delete(self, handoff_id):
        with self._lock:
            self.store.pop(handoff_id, None)

    def exists(self, handoff_id):
        return handoff_id in self.store


class DeviceDictKVStoreBackend(DictKVStoreBackend):
    """In-process dict whose items stay on the device (both runners in one process)."""
    keep_on_device = True


class SharedMemoryKVStoreBackend(KVStoreBackend):
    """Cross-process store; items are addressed by the shm names in their refs."""

    def __init__(self):
        self.records: dict[str, tuple] = {}
        self._own: dict[str, shared_memory.SharedMemory] = {}

    @staticmethod
    def _write(tensor: torch.Tensor) -> SharedMemoryKVRef:
        t = tensor.detach().contiguous().cpu()
        carrier = _CARRIER[t.element_size()]
        arr = t.view(torch.uint8).numpy() if t.element_size() == 1 else \
            t.view({2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()]).numpy().view(carrier)
        nbytes = arr.nbytes
        shm = shared_memory.SharedMemory(create=True, size=max(nbytes, 1), name=f"nvb_kv_{uuid.uuid4().hex[:16]}")
        np.ndarray(arr.shape, dtype=arr.dtype, buffer=shm.buf)[...] = arr
        ref = SharedMemoryKVRef(shm_name=shm.name, shape=tuple(t.shape), dtype=str(t.dtype), nbytes=nbytes)
        shm.close()
        return ref

    @staticmethod
    def _read(ref: SharedMemoryKVRef, unlink: bool) -> torch.Tensor:
        dt = dtype_from_str(ref.dtype)
        esz = torch.empty(0, dtype=dt).element_size()
        shm = shared_memory.SharedMemory(name=ref.shm_name)
        try:
            arr = np.ndarray(ref.shape, dtype=_CARRIER[esz], buffer=shm.buf).copy()
        finally:
            shm.close()
            if unlink:
                try:
                    shared_memory.SharedMemory(name=ref.shm_name).unlink()
                except FileNotFoundError:
                    pass
        t = torch.from_numpy(arr)
        if esz == 1:
            return t.view(torch.uint8).view(dt)
        return t.view({2: torch.int16, 4: torch.int32, 8: torch.int64}[esz]).view(dt)

    def put(self, handoff_id, item):
        ref = self._write(item.kv_blocks)
        sref = self._write(item.scale_blocks) if item.scale_blocks is not None else None
        item.storage_ref, item.scale_storage_ref = ref, sref
        self.records[handoff_id] = (ref, sref, item.num_cached_tokens, item.num_kv_blocks,
                                    item.last_block_num_tokens, item.kv_cache_quant_mode)
        return KVStoreItem(None, None, item.num_cached_tokens, item.num_kv_blocks, item.last_block_num_tokens,
                           item.kv_cache_quant_mode, ref, sref)

    def _load(self, rec, unlink):
        ref, sref, nc, nb, last, mode = rec
        kv = self._read(ref, unlink)
        sc = self._read(sref, unlink) if sref is not None else None
        return KVStoreItem(kv, sc, nc, nb, last, mode, ref, sref)

    def get(self, handoff_id):
        return self._load(self.records[handoff_id], unlink=False)

    def pop(self, handoff_id):
        return self._load(self.records.pop(handoff_id), unlink=True)

    def pop_by_ref(self, ref: SharedMemoryKVRef, scale_ref: SharedMemoryKVRef | None = None, *,
                   num_cached_tokens: int = 0, num_kv_blocks: int = 0, last_block_num_tokens: int = 0,
                   kv_cache_quant_mode: str = "none", unlink: bool = True) -> KVStoreItem:
        kv = self._read(ref, unlink)
        sc = self._read(scale_ref, unlink) if scale_ref is not None else None
        return KVStoreItem(kv, sc, num_cached_tokens, num_kv_blocks, last_block_num_tokens, kv_cache_quant_mode,
                           ref, scale_ref)

    @staticmethod
    def _unlink(ref):
        if ref is None:
            return
        try:
            s = shared_memory.SharedMemory(name=ref.shm_name)
            s.close()
            s.unlink()
        except FileNotFoundError:
            pass

    def delete(self, handoff_id):
        rec = self.records.pop(handoff_id, None)
        if rec is not None:
            self._unlink(rec[0])
            self._unlink(rec[1])

    def delete_by_ref(self, ref):
        if isinstance(ref, SharedMemoryKVRef):
            self._unlink(ref)
        else:
            self.delete(ref)

    def exists(self, handoff_id):
        return handoff_id in self.records


class SyncGpuKVStoreBackend(KVStoreBackend):
    """Device-direct handoff over NCCL point-to-point (the reference's ``sync_gpu``)."""
    device_direct = True

    def __init__(self, rank: int, peer_rank: int | None = None, group=None):
        self.rank = rank
        self.peer_rank = peer_rank
        self.group = group
        self.pending: dict[str, KVStoreItem] = {}

    def set_peer_rank(self, peer_rank: int) -> None:
        self.peer_rank = int(peer_rank)

    def put(self, handoff_id, item):
        if self.peer_rank is None:
            raise RuntimeError("SyncGpuKVStoreBackend needs a peer rank before put()")
        kv = item.kv_blocks
        ref = SyncGpuKVRef(handoff_id=handoff_id, shape=tuple(kv.shape), dtype=str(kv.dtype),
                           nbytes=kv.numel() * kv.element_size(), src_rank=self.rank, dst_rank=self.peer_rank)
        if item.scale_blocks is not None:
            sc = item.scale_blocks
            ref.scale_shape, ref.scale_dtype = tuple(sc.shape), str(sc.dtype)
            ref.scale_nbytes = sc.numel() * sc.element_size()
        item.storage_ref = ref
        self.pending[handoff_id] = item
        return KVStoreItem(None, None, item.num_cached_tokens, item.num_kv_blocks, item.last_block_num_tokens,
                           item.kv_cache_quant_mode, ref, None)

    def _tensors(self, item):
        kv = item.kv_blocks.contiguous()
        if kv.dtype == torch.float8_e4m3fn:  # NCCL has no fp8 type: move the bytes
            kv = kv.view(torch.uint8)
        out = [kv]
        if item.scale_blocks is not None:
            out.append(item.scale_blocks.contiguous())
        return out

    def send_pending(self, handoff_id: str) -> None:
        import torch.distributed as dist
        item = self.pending.pop(handoff_id)
        for t in self._tensors(item):
            dist.send(t, dst=item.storage_ref.dst_rank, group=self.group)

    def submit_send(self, handoff_id: str) -> AsyncSendState:
        import torch.distributed as dist
        item = self.pending.pop(handoff_id)
        ts = self._tensors(item)
        works = [dist.isend(t, dst=item.storage_ref.dst_rank, group=self.group) for t in ts]
        return AsyncSendState(handoff_id, works, ts)

    def _alloc(self, ref: SyncGpuKVRef, device):
        dt = dtype_from_str(ref.dtype)
        kv = torch.empty(ref.shape, dtype=torch.uint8 if dt == torch.float8_e4m3fn else dt, device=device)
        sc = None
        if ref.scale_shape is not None:
            sc = torch.empty(ref.scale_shape, dtype=dtype_from_str(ref.scale_dtype), device=device)
        return kv, sc, dt

    def submit_recv_by_ref(self, ref: SyncGpuKVRef, device, *, num_cached_tokens=0, num_kv_blocks=0,
                           last_block_num_tokens=0, kv_cache_quant_mode="none") -> AsyncRecvState:
        import torch.distributed as dist
        kv, sc, dt = self._alloc(ref, device)
        works = [dist.irecv(kv, src=ref.src_rank, group=self.group)]
        if sc is not None:
            works.append(dist.irecv(sc, src=ref.src_rank, group=self.group))
        item = KVStoreItem(kv.view(dt) if dt == torch.float8_e4m3fn else kv, sc, num_cached_tokens, num_kv_blocks,
                           last_block_num_tokens, kv_cache_quant_mode, ref, None)
        return AsyncRecvState(ref.handoff_id, works, kv, sc, item)

    @staticmethod
    def transfer_done(state) -> bool:
        return all(w.is_completed() for w in state.works)

    @staticmethod
    def wait_transfer(state) -> None:
        for w in state.works:
            w.wait()

    def finish_recv(self, state: AsyncRecvState) -> KVStoreItem:
        self.wait_transfer(state)
        return state.item

    def pop_by_ref(self, ref: SyncGpuKVRef, device="cuda", **kw) -> KVStoreItem:
        st = self.submit_recv_by_ref(ref, device, **kw)
        return self.finish_recv(st)

    def get(self, handoff_id):
        return self.pending[handoff_id]

    def pop(self, handoff_id):
        return self.pending.pop(handoff_id)

    def delete(self, handoff_id):
        self.pending.pop(handoff_id, None)

    def exists(self, handoff_id):
        return handoff_id in self.pending


def make_backend(name: str, **kw) -> KVStoreBackend:
    if name == "dict":
        return DictKVStoreBackend()
    if name == "device":
        return DeviceDictKVStoreBackend()
    if name in ("shared_memory", "shm"):
        return SharedMemoryKVStoreBackend()
    if name == "sync_gpu":
        return SyncGpuKVStoreBackend(**kw)
    raise ValueError(f"unknown KV store backend {name!r}")
