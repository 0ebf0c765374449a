"""Engine configuration.

One immutable-by-convention :class:`EngineConfig` per engine instance; there is no
module-level global that several engines share (the reference mutates a shared
``config`` object in ``nanovllm/engine/llm_engine.py:17-25``).

Field names and defaults follow the reference's ``Config`` dataclass
(``nanovllm/config.py:27-80``) so that a user of the reference finds the same knobs:
``max_model_len``, ``max_num_seqs``, ``num_blocks``, ``block_size``,
``max_num_batched_tokens``, ``enable_chunked_prefill``, ``prefill_chunk_size``,
``kv_cache_dtype``, ``kv_cache_quant_mode``, ``eos`` ...

Differences (all deliberate):

* ``num_blocks=-1`` (the default here) sizes the KV pool from free device memory and
  ``gpu_memory_utilization``; the reference always allocates a fixed 256 blocks.
* ``kv_cache_quant_mode`` accepts ``"fp8"`` (e4m3 with one fp32 scale per block per
  KV head) in addition to the reference's ``"none"`` and ``"int8_mock"``.
* ``comm_backend`` selects the tensor-parallel reduction: ``"fused"`` (peer-memory
  kernels, the product path) or ``"nccl"`` (the reference's behaviour, kept as the
  baseline).
* ``enable_cuda_graph`` defaults to True and is honoured by the runner (the reference
  captures graphs but never replays them, ``nanovllm/engine/model_runner.py:82,534``).
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field

import torch

_DTYPE_ALIASES = {
    "float32": torch.float32,
    "fp32": torch.float32,
    "float": torch.float32,
    "float16": torch.float16,
    "fp16": torch.float16,
    "half": torch.float16,
    "bfloat16": torch.bfloat16,
    "bf16": torch.bfloat16,
    "float8_e4m3fn": torch.float8_e4m3fn,
    "fp8": torch.float8_e4m3fn,
    "fp8_e4m3": torch.float8_e4m3fn,
    "int8": torch.int8,
}


def resolve_torch_dtype(dtype):
    """Map a dtype alias (``"bf16"``, ``"fp32"``, ``"auto"`` ...) to a ``torch.dtype``.

    ``None`` and ``"auto"`` resolve to ``None`` (meaning: inherit), as in the
    reference's ``resolve_torch_dtype`` (``nanovllm/config.py:6-25``).
    """
    if isinstance(dtype, torch.dtype):
        return dtype
    if dtype is None or dtype == "auto":
        return None
    key = str(dtype).lower()
    if key not in _DTYPE_ALIASES:
        raise ValueError(f"unsupported dtype: {dtype}")
    return _DTYPE_ALIASES[key]


KV_QUANT_MODES = ("none", "int8_mock", "fp8")
COMM_BACKENDS = ("fused", "nccl")


@dataclass
class EngineConfig:
    model_path: str | None = None
    # Model architecture override: a preset name ("qwen3-0.6b", "qwen3-8b", "qwen3-32b",
    # "tiny") or a dict of HF config fields. Used when model_path has no checkpoint.
    model: str | dict | None = None
    device: str = "cuda"
    dtype: torch.dtype | str = torch.bfloat16
    kv_cache_dtype: torch.dtype | str | None = "auto"
    attention_compute_dtype: torch.dtype | str | None = "auto"
    kv_cache_quant_mode: str = "none"
    kv_cache_scale_dtype: torch.dtype | str = torch.float32

    max_model_len: int = 4096
    max_num_seqs: int = 256
    num_blocks: int = -1
    block_size: int = 256
    gpu_memory_utilization: float = 0.90
    max_num_batched_tokens: int = 16384
    use_cache: bool = True
    eos: int = -1
    enable_chunked_prefill: bool = False
    prefill_chunk_size: int = 256

    tensor_parallel_size: int = 1
    comm_backend: str = "fused"
    # Fused backend, decode-sized steps (<= 256 tokens): the o_proj / down_proj GEMMs store
    # their output rows at the owner rank (reduce-scatter in the GEMM epilogue) and the owner
    # normalises and all-gathers.  Off by default: on two B200s this path (two cross-GPU
    # handshakes per reduction) measured 27-53 us per o_proj / down_proj against 17-39 us for
    # the GEMM followed by the one-shot all-reduce + residual + RMSNorm kernel (one handshake).
    fused_reduce_scatter: bool = False
    # Sample inside the lm_head GEMM's epilogue (one tensor-parallel rank, no top-p rows in the
    # step): the logits are never written to memory.  Off by default: on a B200 the Qwen3-8B lm_head
    # at 256 tokens takes 326 us either way when greedy (the 78 MB of logits stay in the 126 MB L2,
    # so the sampler kernel after the GEMM costs about 2 us), and with temperature rows the Gumbel
    # noise in the GEMM's four epilogue warps makes it 577 us against 433 us for GEMM + sampler.
    fused_sampler: bool = False
    enable_cuda_graph: bool = True
    cuda_graph_max_bs: int = 512
    enable_prefix_cache: bool = True
    enable_preemption: bool = True
    # Reference quirk (nanovllm/layers/sampler.py:33-43): if any temperature in the batch
    # is <= 0 the whole batch is sampled greedily. Off by default: per-row sampling.
    batch_greedy_compat: bool = False
    seed: int = 0
    # Random-init (no checkpoint) weight std, N(0, init_std).
    init_std: float = 0.02
    # Use the hand-written CUDA ops (True) or the torch reference ops (False, CPU/oracle).
    use_custom_kernels: bool | None = None
    enforce_eager: bool = False
    # GEMM plans from the shape alone instead of timing (identical numerics in every process:
    # P/D pairs and TP groups reproduce a monolithic run bit for bit); also NVB_DETERMINISTIC=1
    deterministic: bool = False
    # Allocate the KV pool with cudaMalloc + CUDA IPC so another process can push blocks
    # into it (the decode side of the NVLink P/D push).
    kv_pool_ipc: bool = False
    # Prefill attention kernel over bf16 KV: "tcgen05" (TMEM accumulators, the default) or "mma"
    # (the mma.sync kernel, which fp8 KV always uses).  The reference's per-layer backend switch
    # (nanovllm/layers/attention.py:58, forward_backend) made a config field.
    prefill_attention: str = "tcgen05"
    # Timeout of the tensor-parallel process group: a collective whose peer never joins (a rank
    # that died or stalls between steps) ends with an error after this long instead of waiting.
    dist_timeout_s: float = 600.0
    # Append every generate call's metrics (the ``return_metrics`` dict without the block-usage
    # snapshot, plus a timestamp) as one JSON line to this file; rank 0 only.
    metrics_path: str | None = None
    extra: dict = field(default_factory=dict)

    def __post_init__(self):
        self.dtype = resolve_torch_dtype(self.dtype) or torch.bfloat16
        self.attention_compute_dtype = resolve_torch_dtype(self.attention_compute_dtype) or self.dtype
        self.kv_cache_scale_dtype = resolve_torch_dtype(self.kv_cache_scale_dtype) or torch.float32
        if self.kv_cache_quant_mode not in KV_QUANT_MODES:
            raise ValueError(f"unsupported kv_cache_quant_mode: {self.kv_cache_quant_mode}")
        if self.comm_backend not in COMM_BACKENDS:
            raise ValueError(f"unsupported comm_backend: {self.comm_backend}")
        if self.prefill_attention not in ("tcgen05", "mma"):
            raise ValueError(f"unsupported prefill_attention: {self.prefill_attention}")
        kv = resolve_torch_dtype(self.kv_cache_dtype)
        if self.kv_cache_quant_mode == "int8_mock":
            kv = torch.int8
        elif self.kv_cache_quant_mode == "fp8":
            kv = torch.float8_e4m3fn
        elif kv in (torch.float8_e4m3fn,):
            self.kv_cache_quant_mode = "fp8"
        self.kv_cache_dtype = kv or self.dtype
        if self.block_size <= 0 or (self.block_size & (self.block_size - 1)) != 0:
            raise ValueError(f"block_size must be a power of two, got {self.block_size}")
        if self.max_num_seqs <= 0 or self.max_num_batched_tokens <= 0:
            raise ValueError("max_num_seqs and max_num_batched_tokens must be positive")
        if self.tensor_parallel_size not in (1, 2, 4, 8):
            raise ValueError("tensor_parallel_size must be 1, 2, 4 or 8")

    @property
    def is_cuda(self) -> bool:
        return str(self.device).startswith("cuda")

    def replace(self, **kw) -> "EngineConfig":
        return dataclasses.replace(self, **kw)


# Name kept for users of the reference (``nanovllm.config.Config``).
Config = EngineConfig
