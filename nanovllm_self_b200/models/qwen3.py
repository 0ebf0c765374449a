"""Qwen3 dense decoder for the serving engine.

Same math as the reference model (``nanovllm/models/qwen3.py:18-143`` decoder layer,
``:241-510`` model): pre-norm blocks with GQA attention, per-head q/k RMSNorm, NeoX
RoPE, SwiGLU MLP, final RMSNorm, logits only for the last token of each sampling
sequence (``:497-506``).

B200-first layout (not the reference's module-per-projection layout):

* q/k/v are one ``[(Hq + 2 Hkv) * D, H]`` weight -> one GEMM; gate/up are one
  ``[2 I, H]`` weight -> one GEMM whose output feeds the SiLU-and-mul kernel;
* q/k RMSNorm + RoPE + KV-cache store are one kernel over the QKV GEMM output;
* residual add + RMSNorm are one kernel; under tensor parallelism that kernel also
  performs the all-reduce of the row-parallel GEMM output (fused comm backend), and on
  decode-sized steps the reduce-scatter half of it moves into the o_proj / down_proj GEMM
  epilogue (each output row stored at its owner rank), the owner then normalises and
  all-gathers;
* the embedding table and lm_head are vocab-parallel under TP (the reference keeps
  full replicas on every rank, ``:255-258,285``);
* the final norm runs only on the rows that are sampled.

Ops are supplied by an ops object (``ops.get_ops(device)``): hand-written CUDA kernels
on GPU, the plain-PyTorch oracle on CPU.
"""
from __future__ import annotations

import torch

from ..ops import torch_ref
from .configs import Qwen3Arch


class Qwen3Layer:
    __slots__ = ("ln1", "ln2", "qkv", "q_norm", "k_norm", "o", "gate_up", "down")

    def __init__(self):
        for s in self.__slots__:
            setattr(self, s, None)

    def tensors(self) -> dict:
        return {s: getattr(self, s) for s in self.__slots__}


class Qwen3ForCausalLM:
    def __init__(self, arch: Qwen3Arch, tp_rank: int = 0, tp_size: int = 1,
                 dtype: torch.dtype = torch.bfloat16, device="cpu"):
        a = arch
        if a.num_attention_heads % tp_size or a.num_key_value_heads % tp_size or a.intermediate_size % tp_size:
            raise ValueError(f"heads/kv_heads/intermediate must be divisible by tp={tp_size}")
        self.arch = a
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self.dtype = dtype
        self.device = torch.device(device)
        self.num_layers = a.num_hidden_layers
        self.hidden_size = a.hidden_size
        self.head_dim = a.head_dim
        self.num_heads = a.num_attention_heads // tp_size
        self.num_kv_heads = a.num_key_value_heads // tp_size
        self.local_num_kv_heads = self.num_kv_heads
        self.intermediate = a.intermediate_size // tp_size
        self.vocab_size = a.vocab_size
        self.vocab_per_rank = (a.vocab_size + tp_size - 1) // tp_size
        self.vocab_start = tp_rank * self.vocab_per_rank
        self.vocab_end = min(a.vocab_size, self.vocab_start + self.vocab_per_rank)
        self.eps = a.rms_norm_eps
        self.scale = torch_ref.softmax_scale(a.head_dim)
        self.embed: torch.Tensor | None = None
        self.lm_head: torch.Tensor | None = None
        self.norm: torch.Tensor | None = None
        self.layers = [Qwen3Layer() for _ in range(self.num_layers)]
        self.cos_sin = None
        self.ops = None
        self.comm = None

    # ------------------------------------------------------------------ setup
    def finalize(self, ops, comm=None, max_position: int | None = None):
        a = self.arch
        mp = max_position or a.max_position_embeddings
        self.cos_sin = torch_ref.rope_cos_sin(a.head_dim, mp, a.rope_theta, device=self.device)
        self.ops = ops
        self.comm = comm
        return self

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    def weight_bytes(self) -> int:
        n = sum(t.numel() * t.element_size() for L in self.layers for t in L.tensors().values())
        n += self.embed.numel() * self.embed.element_size() + self.norm.numel() * self.norm.element_size()
        if self.lm_head is not self.embed:
            n += self.lm_head.numel() * self.lm_head.element_size()
        return n

    # ---------------------------------------------------------------- forward
    def _reduce_in(self, T):
        """Output buffer for a row-parallel GEMM: the comm layer's symmetric input under TP."""
        if self.comm is not None and self.tp_size > 1:
            return self.comm.input_buffer(T)
        return None

    def _reduce_norm(self, h, residual, w):
        """residual' = allreduce(h) + residual; return (rmsnorm(residual'), residual')."""
        if self.comm is not None and self.tp_size > 1:
            return self.comm.allreduce_add_rmsnorm(h, residual, w, self.eps)
        return self.ops.add_rmsnorm(h, residual, w, self.eps)

    def _rs(self, T: int, k: int) -> bool:
        """Row-parallel GEMMs of this step store their rows at the owner rank (decode steps)."""
        return self.comm is not None and self.tp_size > 1 and self.comm.rs_ok(T, k)

    def forward_hidden(self, input_ids: torch.Tensor, positions: torch.Tensor, ctx, kv_caches, kv_scales=None):
        """Run embedding + all layers.

        Returns (h, residual, normed): with ``normed`` False, h and residual are the last
        layer's output before the final norm (the final norm then runs on the sampled rows
        only); with ``normed`` True (tensor-parallel decode steps, whose row-parallel GEMMs
        reduce-scatter in their epilogue) h already holds the final-normed rows of every token.
        """
        ops = self.ops
        T = input_ids.shape[0]
        if self.comm is not None and self.tp_size > 1:
            self.comm.begin_forward()
        h = ops.embedding(input_ids, self.embed, self.vocab_start)
        residual = None
        nq, nkv, d = self.num_heads, self.num_kv_heads, self.head_dim
        rs = self._rs(T, nq * d) and self._rs(T, self.intermediate)
        n = len(self.layers)
        x = None
        for i, L in enumerate(self.layers):
            if not rs or i == 0:
                x, residual = self._reduce_norm(h, residual, L.ln1)
            qkv = ops.linear(x, L.qkv)
            kc, vc = kv_caches[i]
            ks, vs = kv_scales[i] if kv_scales is not None else (None, None)
            q = ops.qkv_post(qkv, L.q_norm, L.k_norm, self.eps, positions, self.cos_sin, kc, vc,
                             ctx.slot_mapping, ks, vs, nq, nkv, d)
            o = ops.attention(q, kc, vc, ctx, self.scale, ks, vs)
            if rs:
                x, residual = self.comm.linear_rs_norm(o.view(T, nq * d), L.o, L.ln2, self.eps)
            else:
                h = ops.linear(o.view(T, nq * d), L.o, out=self._reduce_in(T))
                x, residual = self._reduce_norm(h, residual, L.ln2)
            a = ops.linear_silu(x, L.gate_up)  # silu(gate) * up, fused into the GEMM epilogue
            if rs:
                # the next layer's ln1, or the final norm after the last layer
                w_next = self.layers[i + 1].ln1 if i + 1 < n else self.norm
                x, residual = self.comm.linear_rs_norm(a, L.down, w_next, self.eps)
            else:
                h = ops.linear(a, L.down, out=self._reduce_in(T))
        if rs:
            return x, residual, True
        return h, residual, False

    def compute_logits(self, h, residual, logits_indices: torch.Tensor, normed: bool = False) -> torch.Tensor:
        """Final norm on the sampled rows only, then the (vocab-parallel) lm_head."""
        if logits_indices.numel() == 0:
            return torch.empty(0, self.vocab_end - self.vocab_start, device=h.device, dtype=torch.float32)
        return self.ops.linear(self.final_rows(h, residual, logits_indices, normed), self.lm_head)

    def final_rows(self, h, residual, logits_indices: torch.Tensor, normed: bool = False) -> torch.Tensor:
        """The final-normed hidden rows of the sampled tokens (the lm_head's input)."""
        ops = self.ops
        # every row sampled (decode steps: one token per sequence, indices 0..T-1): no gather
        every_row = logits_indices.numel() == h.shape[0]
        if normed:
            x = h if every_row else h.index_select(0, logits_indices)
        elif self.comm is not None and self.tp_size > 1:
            hs = h if every_row else h.index_select(0, logits_indices)
            rs = residual if every_row else residual.index_select(0, logits_indices)
            x, _ = self.comm.allreduce_add_rmsnorm(hs, rs, self.norm, self.eps, final=True)
        else:
            x, _ = ops.add_rmsnorm_rows(h, residual, self.norm, self.eps, logits_indices)
        return x

    def forward(self, input_ids, positions, ctx, kv_caches, kv_scales=None):
        h, residual, normed = self.forward_hidden(input_ids, positions, ctx, kv_caches, kv_scales)
        return self.compute_logits(h, residual, ctx.logits_indices, normed)
