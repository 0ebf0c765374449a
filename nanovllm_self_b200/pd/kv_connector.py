"""KV connector: export a finished prefill's KV blocks, hand them to a store, import them on decode.

Reference: ``pd_self/kv_connector.py:25-326``.  Same roles and methods:

* producer: ``save_kv(seq) -> KVTransferMeta`` gathers ``kv_cache[:, :, block_table[:n]]``
  for ``n = ceil(num_cached_tokens / block_size)`` (and the scale blocks of a quantised
  cache), puts it in the backend and returns light metadata; ``flush_kv_transfer(meta)``
  triggers the send of device-direct backends;
* consumer: ``load_kv(meta, dst_block_ids)`` fetches the item and ``load_kv_item`` writes it
  into the local pool; ``discard(meta)`` drops an unused handoff.

Differences: the gather and the scatter are single vectorised index operations on the
device (the reference issues one ``copy_`` per destination block, :299-309), and KV that
crosses devices inside one process goes device-to-device without a host round trip.
``handoff_id = engine_id:seq_idx:num_cached:uuid8`` as in the reference (:39-50).
"""
from __future__ import annotations

import uuid

import torch

from .kv_store import KVStoreBackend, KVStoreItem, SharedMemoryKVStoreBackend
from .payload import KVTransferMeta, SharedMemoryKVRef, SyncGpuKVRef


def _raw(t: torch.Tensor) -> torch.Tensor:
    """Byte view of fp8 tensors (index ops and NCCL have no fp8 kernels/types)."""
    return t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t


class KVConnector:
    def __init__(self, config, role: str, engine_id: str, kv_store_backend: KVStoreBackend, export: bool = True):
        if role not in ("producer", "consumer"):
            raise ValueError("role must be 'producer' or 'consumer'")
        # export=False: metadata only (the KV is pushed straight from the pool by a kernel)
        self.export = export
        self.config = config
        self.role = role
        self.engine_id = engine_id
        self.kv_store_backend = kv_store_backend
        self.model_runner = None

    def register_model_runner(self, model_runner) -> None:
        self.model_runner = model_runner

    # ---------------------------------------------------------------- producer
    def _build_handoff_id(self, seq) -> str:
        return f"{self.engine_id}:{seq.seq_idx}:{seq.num_cached_tokens}:{uuid.uuid4().hex[:8]}"

    def _last_block_num_tokens(self, num_cached: int) -> int:
        if num_cached == 0:
            return 0
        bs = self.config.block_size
        rem = num_cached % bs
        return bs if rem == 0 else rem

    def _export_kv_snapshot(self, seq):
        r = self.model_runner
        n_cached = seq.num_cached_tokens
        if n_cached == 0:
            return None, None, 0, 0, []
        bs = self.config.block_size
        n = (n_cached + bs - 1) // bs
        src = list(seq.block_table[:n])
        idx = torch.as_tensor(src, dtype=torch.long, device=r.kv_cache.device)
        kv = _raw(r.kv_cache).index_select(2, idx)
        if r.kv_cache.dtype == torch.float8_e4m3fn:
            kv = kv.view(torch.float8_e4m3fn)
        sc = r.kv_scale_cache.index_select(2, idx) if r.kv_scale_cache is not None else None
        b = self.kv_store_backend
        if not (b.device_direct or getattr(b, "keep_on_device", False)):
            kv = kv.cpu()
            sc = sc.cpu() if sc is not None else None
        return kv, sc, n, self._last_block_num_tokens(n_cached), src

    def save_kv(self, seq) -> KVTransferMeta:
        if self.role != "producer":
            raise RuntimeError("save_kv is a producer operation")
        if self.export:
            kv, sc, n, last, src = self._export_kv_snapshot(seq)
        else:
            bs = self.config.block_size
            n = (seq.num_cached_tokens + bs - 1) // bs
            kv, sc, last, src = None, None, self._last_block_num_tokens(seq.num_cached_tokens), list(seq.block_table[:n])
        hid = self._build_handoff_id(seq)
        mode = self.config.kv_cache_quant_mode
        meta = KVTransferMeta(handoff_id=hid, producer_id=self.engine_id, num_cached_tokens=seq.num_cached_tokens,
                              num_kv_blocks=n, last_block_num_tokens=last, src_block_table=src,
                              kv_cache_quant_mode=mode)
        if kv is None:
            return meta
        stored = self.kv_store_backend.put(hid, KVStoreItem(kv, sc, seq.num_cached_tokens, n, last, mode))
        if stored is not None:
            meta.storage_ref = stored.storage_ref
            meta.scale_storage_ref = stored.scale_storage_ref
        return meta

    def flush_kv_transfer(self, transfer_meta: KVTransferMeta) -> None:
        b = self.kv_store_backend
        if hasattr(b, "send_pending") and b.exists(transfer_meta.handoff_id):
            b.send_pending(transfer_meta.handoff_id)

    # ---------------------------------------------------------------- consumer
    def load_kv(self, transfer_meta: KVTransferMeta, dst_block_ids: list) -> None:
        if transfer_meta.num_kv_blocks == 0:
            return
        b = self.kv_store_backend
        ref = transfer_meta.storage_ref
        if isinstance(ref, SharedMemoryKVRef) and isinstance(b, SharedMemoryKVStoreBackend):
            item = b.pop_by_ref(ref, transfer_meta.scale_storage_ref, num_cached_tokens=transfer_meta.num_cached_tokens,
                                num_kv_blocks=transfer_meta.num_kv_blocks,
                                last_block_num_tokens=transfer_meta.last_block_num_tokens,
                                kv_cache_quant_mode=transfer_meta.kv_cache_quant_mode)
            b.records.pop(transfer_meta.handoff_id, None)
        elif isinstance(ref, SyncGpuKVRef) and hasattr(b, "pop_by_ref"):
            item = b.pop_by_ref(ref, device=self.model_runner.kv_cache.device,
                                num_cached_tokens=transfer_meta.num_cached_tokens,
                                num_kv_blocks=transfer_meta.num_kv_blocks,
                                last_block_num_tokens=transfer_meta.last_block_num_tokens,
                                kv_cache_quant_mode=transfer_meta.kv_cache_quant_mode)
        else:
            item = b.pop(transfer_meta.handoff_id)
        self.load_kv_item(item, dst_block_ids)

    def load_kv_item(self, item: KVStoreItem, dst_block_ids: list) -> None:
        r = self.model_runner
        n = item.num_kv_blocks
        if n == 0:
            return
        if len(dst_block_ids) < n:
            raise ValueError(f"need {n} destination blocks, got {len(dst_block_ids)}")
        dev = r.kv_cache.device
        idx = torch.as_tensor(list(dst_block_ids[:n]), dtype=torch.long, device=dev)
        kv = item.kv_blocks.to(dev, non_blocking=True)
        if kv.dtype != r.kv_cache.dtype:
            if kv.dtype == torch.uint8:
                kv = kv.view(r.kv_cache.dtype)
            else:
                raise TypeError(f"KV dtype {kv.dtype} does not match the pool ({r.kv_cache.dtype})")
        _raw(r.kv_cache).index_copy_(2, idx, _raw(kv))
        if item.scale_blocks is not None and r.kv_scale_cache is not None:
            r.kv_scale_cache.index_copy_(2, idx, item.scale_blocks.to(dev, non_blocking=True))

    def discard(self, transfer_meta: KVTransferMeta | None) -> None:
        if transfer_meta is None:
            return
        b = self.kv_store_backend
        ref = transfer_meta.storage_ref
        if ref is not None and hasattr(b, "delete_by_ref"):
            b.delete_by_ref(ref)
        if transfer_meta.scale_storage_ref is not None and hasattr(b, "delete_by_ref"):
            b.delete_by_ref(transfer_meta.scale_storage_ref)
        b.delete(transfer_meta.handoff_id)
