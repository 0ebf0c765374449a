"""Handoff records passed from the prefill side to the decode side.

Field-for-field the same contract as the reference (``pd_self/payload.py:7-98``), because
these records cross process boundaries (pickled payload files) and a reader of one side
must understand the other: ``HandoffPayload.token_ids`` holds the prompt plus the first
generated token, and ``num_cached_tokens`` counts only the tokens whose KV was written
(it excludes that first generated token).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional


@dataclass
class SyncGpuKVRef:
    """Reference to a KV tensor sent GPU-to-GPU over NCCL point-to-point."""
    handoff_id: str
    shape: tuple
    dtype: str
    nbytes: int
    src_rank: int
    dst_rank: int
    scale_shape: tuple | None = None
    scale_dtype: str | None = None
    scale_nbytes: int = 0


@dataclass
class SharedMemoryKVRef:
    """Everything another process needs to attach to a POSIX shared-memory KV blob."""
    shm_name: str
    shape: tuple
    dtype: str
    nbytes: int


@dataclass
class DevicePushRef:
    """KV already written into the consumer's pool by the fused push kernel."""
    handoff_id: str
    dst_block_ids: List[int]
    done: bool = True


@dataclass
class KVTransferMeta:
    handoff_id: str
    producer_id: str
    num_cached_tokens: int
    num_kv_blocks: int
    last_block_num_tokens: int
    src_block_table: List[int] = field(default_factory=list)  # trace/debug only
    storage_ref: Optional[object] = None
    scale_storage_ref: Optional[object] = None
    kv_cache_quant_mode: str = "none"


@dataclass
class HandoffPayload:
    seq_idx: int
    request_id: str
    token_ids: List[int]
    num_prompt_tokens: int
    num_cached_tokens: int
    temperature: float
    max_tokens: int
    ignore_eos: bool
    finished: bool
    transfer_meta: Optional[KVTransferMeta] = None
    session_id: Optional[str] = None
    top_p: float = 1.0
    prefix_cache_hit: bool = False
    prefix_cached_tokens: int = 0
    prefix_cache_source: Optional[str] = None
