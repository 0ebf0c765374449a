"""Prefill/decode (P/D) disaggregation: separate prefill and decode engines with a KV handoff.

Reference: ``pd_self/`` (payloads, KV stores, connector, engines, offline and online
coordinators, multiprocess workers, control plane, agent-aware router).
"""
from .payload import HandoffPayload, KVTransferMeta, SharedMemoryKVRef, SyncGpuKVRef
from .request_state import RequestState, RequestStatus, TokenEvent
from .runtime_types import DecodeStepOutput, OnlineSchedulerStepMetrics

__all__ = ["HandoffPayload", "KVTransferMeta", "SharedMemoryKVRef", "SyncGpuKVRef", "RequestState", "RequestStatus",
           "TokenEvent", "DecodeStepOutput", "OnlineSchedulerStepMetrics"]
