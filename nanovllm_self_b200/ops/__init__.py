"""Op sets used by the model.

``get_ops(device)`` returns the op set for a device:

* CUDA device -> :class:`nanovllm_self_b200.ops.cuda_ops.CudaOps`, the hand-written
  sm_100a kernels of the in-tree extension ``nanovllm_self_b200._C``.  If that
  extension is missing or was not built for sm_100a, this raises: there is no silent
  fallback on a GPU.
* CPU -> :class:`TorchOps`, the plain-PyTorch oracle (used by the tiny CPU model and
  by every kernel test as the fp32 reference).
"""
from __future__ import annotations

import torch

from . import torch_ref as R


class TorchOps:
    name = "torch"

    def embedding(self, ids, w, vocab_start=0):
        return R.embedding(ids, w, vocab_start)

    def add_rmsnorm(self, x, residual, w, eps):
        return R.add_rmsnorm(x, residual, w, eps)

    def add_rmsnorm_rows(self, h, residual, w, eps, rows):
        idx = rows.long()
        return R.add_rmsnorm(h.index_select(0, idx), residual.index_select(0, idx), w, eps)

    def rmsnorm(self, x, w, eps):
        return R.rmsnorm(x, w, eps)

    def linear(self, x, w, out=None):
        y = R.linear(x, w)
        if out is not None:
            out.copy_(y)
            return out
        return y

    def qkv_post(self, qkv, q_norm, k_norm, eps, positions, cos_sin, k_cache, v_cache, slot_mapping,
                 k_scale, v_scale, nq, nkv, d):
        T = qkv.shape[0]
        q = qkv[:, :nq * d].reshape(T, nq, d)
        k = qkv[:, nq * d:(nq + nkv) * d].reshape(T, nkv, d)
        v = qkv[:, (nq + nkv) * d:].reshape(T, nkv, d)
        q = R.apply_rope(R.rmsnorm(q, q_norm, eps), positions, cos_sin)
        k = R.apply_rope(R.rmsnorm(k, k_norm, eps), positions, cos_sin)
        R.store_kv(k, v, k_cache, v_cache, slot_mapping, k_scale, v_scale)
        return q

    def attention(self, q, k_cache, v_cache, ctx, scale, k_scale=None, v_scale=None):
        q_lens = ctx.host_q_lens
        k_lens = ctx.host_k_lens
        bt = ctx.block_tables.tolist()
        return R.paged_attention(q, k_cache, v_cache, q_lens, k_lens, bt, scale, k_scale, v_scale)

    def silu_mul(self, x):
        return R.silu_mul(x)

    def linear_silu(self, x, w_gate_up):
        """silu(gate) * up of x @ w^T, w in the interleaved gate/up layout."""
        return R.silu_mul_interleaved(R.linear(x, w_gate_up)).to(x.dtype)

    def sample(self, logits, temperatures, top_p=None, seeds=None, step=0, batch_greedy_compat=False,
               generator=None, use_top_p=True, col_offset=0):
        return R.sample(logits, temperatures, top_p, generator, batch_greedy_compat).to(torch.int32)


_TORCH_OPS = TorchOps()


def get_ops(device, use_custom_kernels: bool | None = None):
    dev = torch.device(device)
    if dev.type == "cuda" and use_custom_kernels is not False:
        from .cuda_ops import CudaOps
        return CudaOps()
    return _TORCH_OPS
