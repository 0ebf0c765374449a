"""Op set backed by the hand-written sm_100a kernels (``nanovllm_self_b200._C``).

Every method launches the extension's kernels on the current stream; scratch buffers
(split-K partials, split-KV partials, sampler partials) are allocated once per device
and reused, so the ops are CUDA-graph capturable.
"""
from __future__ import annotations

import torch

from . import torch_ref as R
from ._ext import load

_GEMM_WS_ELEMS = 24 << 20        # fp32 stream-K partial tiles (96 MiB: 2 per CTA of up to 256 x 256)
_GEMM_COUNTERS = 1 << 16         # split-K arrival counters (4 per output tile)
_ATTN_PART_ROWS = 1 << 16        # (seq, q head, split) rows of split-KV scratch
_SAMPLE_PART = 1 << 16
_SAMPLE_KEYS = 4096              # rows of one fused lm_head + sampler call


class _Scratch:
    def __init__(self, device):
        self.gemm = torch.empty(_GEMM_WS_ELEMS, dtype=torch.float32, device=device)
        self.gemm_counters = torch.zeros(_GEMM_COUNTERS, dtype=torch.int32, device=device)
        self.part_o = torch.empty(_ATTN_PART_ROWS * 128, dtype=torch.float32, device=device)
        self.part_lse = torch.empty(_ATTN_PART_ROWS, dtype=torch.float32, device=device)
        self.sample_val = torch.empty(_SAMPLE_PART, dtype=torch.float32, device=device)
        self.sample_idx = torch.empty(_SAMPLE_PART, dtype=torch.int32, device=device)
        self.sample_keys = torch.zeros(_SAMPLE_KEYS, dtype=torch.int64, device=device)  # zero between calls


class CudaOps:
    name = "cuda-sm100a"

    def __init__(self):
        self.C = load()
        self._scratch: dict = {}
        self.num_sms = {}
        # Number of kernels this op set has launched (graph replays are added by the runner).
        self.launches = 0
        self._plans: dict = {}
        self.last_plan = None
        # prefill attention on the tcgen05 kernel (bf16 KV); False: the mma.sync kernel
        self.prefill_tc = True

    def scratch(self, device) -> _Scratch:
        key = torch.device(device).index
        s = self._scratch.get(key)
        if s is None:
            s = _Scratch(device)
            self._scratch[key] = s
            self.num_sms[key] = torch.cuda.get_device_properties(device).multi_processor_count
        return s

    # ----------------------------------------------------------- elementwise
    def embedding(self, ids, w, vocab_start=0):
        out = torch.empty(ids.shape[0], w.shape[1], dtype=w.dtype, device=w.device)
        self.C.embedding(ids, w, int(vocab_start), out)
        self.launches += 1
        return out

    def add_rmsnorm(self, x, residual, w, eps):
        out = torch.empty(x.shape[0], x.shape[1], dtype=x.dtype, device=x.device)
        if residual is None:
            self.C.add_rmsnorm(x, None, None, w, out, float(eps), None)
            self.launches += 1
            return out, x
        self.C.add_rmsnorm(x, residual, residual, w, out, float(eps), None)
        self.launches += 1
        return out, residual

    def add_rmsnorm_rows(self, h, residual, w, eps, rows):
        """Norm of (h + residual) at row indices ``rows`` only (final norm before lm_head)."""
        out = torch.empty(rows.shape[0], h.shape[1], dtype=h.dtype, device=h.device)
        res_out = torch.empty_like(out)
        self.C.add_rmsnorm(h, residual, res_out, w, out, float(eps), rows)
        self.launches += 1
        return out, res_out

    def rmsnorm(self, x, w, eps):
        return self.add_rmsnorm(x, None, w, eps)[0]

    def silu_mul(self, x):
        out = torch.empty(x.shape[0], x.shape[1] // 2, dtype=x.dtype, device=x.device)
        self.C.silu_mul(x, out)
        self.launches += 1
        return out

    # ----------------------------------------------------------------- GEMM
    def linear(self, x, w, out=None):
        if out is None:
            out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
        if x.shape[0] == 0:
            return out
        sc = self.scratch(x.device)
        self.last_plan = self.C.linear_tuned(x, w, out, sc.gemm, sc.gemm_counters)
        self.launches += 1
        return out

    def linear_silu(self, x, w_gate_up):
        """silu(gate) * up of x @ w^T in one GEMM (SiLU-and-mul epilogue); w's rows are in the
        interleaved gate/up layout of ``torch_ref.interleave_gate_up``."""
        out = torch.empty(x.shape[0], w_gate_up.shape[0] // 2, dtype=x.dtype, device=x.device)
        if x.shape[0] == 0:
            return out
        sc = self.scratch(x.device)
        self.last_plan = self.C.linear_tuned(x, w_gate_up, out, sc.gemm, sc.gemm_counters, 1)
        self.launches += 1
        return out

    def _plan(self, m, n, k):
        key = (m, n, k)
        p = self._plans.get(key)
        if p is None:
            p = self._plans[key] = self.C.gemm_plan(m, n, k)
        return p

    # ------------------------------------------------------------ attention
    def qkv_post(self, qkv, q_norm, k_norm, eps, positions, cos_sin, k_cache, v_cache, slot_mapping,
                 k_scale, v_scale, nq, nkv, d):
        q = torch.empty(qkv.shape[0], nq * d, dtype=qkv.dtype, device=qkv.device)
        self.C.qkv_post(qkv, q, q_norm, k_norm, float(eps), positions, cos_sin, k_cache, v_cache,
                        k_scale, v_scale, slot_mapping, nq, nkv)
        self.launches += 1
        return q

    def attention(self, q, k_cache, v_cache, ctx, scale, k_scale=None, v_scale=None):
        T = q.shape[0]
        nkv, d = k_cache.shape[1], k_cache.shape[3]
        nq = q.shape[1] // d if q.dim() == 2 else q.shape[1]
        out = torch.empty(T, nq * d, dtype=q.dtype, device=q.device)
        nd, B = ctx.num_decode_seqs, ctx.num_seqs
        sc = self.scratch(q.device)
        if nd > 0:
            sms = self.num_sms[q.device.index]
            splits = int(self.C.decode_splits(nd, nkv, max(1, ctx.max_seqlen_k), sms))
            while splits > 1 and nd * nq * splits > sc.part_lse.numel():
                splits //= 2
            self.C.attn_decode(q, k_cache, v_cache, k_scale, v_scale, ctx.block_tables, ctx.cu_seqlens_q,
                               ctx.context_lens, out, sc.part_o, sc.part_lse, nq, nkv, splits, 0, nd, float(scale))
            self.launches += 2 if splits > 1 else 1
        if B > nd:
            self.C.attn_prefill(q, k_cache, v_cache, k_scale, v_scale, ctx.block_tables, ctx.cu_seqlens_q,
                                ctx.context_lens, out, nq, nkv, nd, B - nd, max(1, ctx.max_seqlen_q), float(scale),
                                int(self.prefill_tc))
            self.launches += 1
        return out

    # -------------------------------------------------------------- sampling
    sample_keys_cap = _SAMPLE_KEYS

    def lm_head_sample(self, x, w, temperatures, step, col_offset=0):
        """Tokens sampled from x @ w^T (greedy where the temperature is <= 0, else Gumbel-max at
        it) by the lm_head GEMM's sampling epilogue: the logits are never written to memory.
        Same draws as ``linear`` followed by ``sample`` (same bf16 logits, same noise)."""
        rows = x.shape[0]
        tok = torch.empty(rows, dtype=torch.int32, device=x.device)
        if rows == 0:
            return tok
        sc = self.scratch(x.device)
        self.last_plan = self.C.linear_sample(x, w, sc.sample_keys, temperatures, step, int(col_offset), tok, None,
                                              sc.gemm, sc.gemm_counters, True)
        self.launches += 2
        return tok

    def sample(self, logits, temperatures, top_p=None, seeds=None, step=None, batch_greedy_compat=False,
               generator=None, use_top_p=False, col_offset=0):
        rows, V = logits.shape
        if use_top_p:
            # one CTA per row: nucleus threshold by a two-level mass histogram, then Gumbel-max
            # over the nucleus (no sort, no host sync); batch_greedy_compat is applied by the runner
            tok = torch.empty(rows, dtype=torch.int32, device=logits.device)
            tp = top_p.float() if top_p is not None else None
            self.C.sample_rows(logits, int(col_offset), temperatures, tp, step, tok, None)
            self.launches += 1
            return tok
        sc = self.scratch(logits.device)
        nchunk = int(self.C.sample_chunks(rows, V))
        tok = torch.empty(rows, dtype=torch.int32, device=logits.device)
        self.C.sample(logits, int(col_offset), temperatures, step, sc.sample_val, sc.sample_idx, nchunk, tok, None)
        self.launches += 2
        return tok

    def sample_partial(self, logits, temperatures, step, col_offset):
        """(best score, global token id) per row over this shard's columns."""
        rows, V = logits.shape
        sc = self.scratch(logits.device)
        nchunk = int(self.C.sample_chunks(rows, V))
        tok = torch.empty(rows, dtype=torch.int32, device=logits.device)
        val = torch.empty(rows, dtype=torch.float32, device=logits.device)
        self.C.sample(logits, int(col_offset), temperatures, step, sc.sample_val, sc.sample_idx, nchunk, tok, val)
        self.launches += 2
        return val, tok
