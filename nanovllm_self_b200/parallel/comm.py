"""Tensor-parallel communication for the model.

The reference reduces the row-parallel o_proj/down_proj outputs with an in-place NCCL
``all_reduce`` (``nanovllm/distributed/parallel_state.py:62-71``, called at
``nanovllm/models/qwen3.py:124,138``) and keeps the embedding and lm_head replicated.

Here every reduction is fused with what follows it:

* ``linear_rs_norm(x, w, w_norm)`` (decode-sized steps): the row-parallel GEMM stores each
  output row straight into the memory of the rank that owns it (reduce-scatter in the GEMM
  epilogue, NVLink peer stores); the owner sums the partials, adds the residual,
  RMS-normalises and all-gathers the rows by peer stores, in one kernel.
* ``allreduce_add_rmsnorm(h, residual, w)``: sum the per-rank partial ``h`` over the TP
  group, add the residual, RMS-normalise.  Backend ``"fused"`` does all three in ONE
  kernel that reads the peers' partials straight from their HBM over NVLink (symmetric
  buffers, see :mod:`nanovllm_self_b200.parallel.symm`); backend ``"nccl"`` is the
  reference's behaviour (NCCL all-reduce, then the local add+norm kernel) and is kept
  as the measured baseline.
* ``vocab_parallel_sample``: each rank holds ``V / tp`` logits; one sampler kernel per
  step reduces the shard and combines it with the other ranks' inside the kernel (per-row
  (score, token) pairs, and for top-p the maxima and mass histograms, by peer stores into
  the symmetric buffer); greedy, temperature and top-p, graph-capturable, no NCCL.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .state import TPState


class TPComm:
    def __init__(self, tp: TPState, backend: str = "fused", config=None):
        self.tp = tp
        self.backend = backend
        self.config = config
        self.runner = None
        self.symm = None
        self.ops = None
        self.launches = 0
        # GEMM -> reduce-scatter path for decode-sized steps (fused backend only)
        self.rs_enabled = bool(getattr(config, "fused_reduce_scatter", False)) if config is not None else False

    def bind(self, runner):
        self.runner = runner
        self.ops = runner.ops
        if self.backend == "fused" and runner.is_cuda:
            from .symm import SymmetricWorkspace
            c = runner.config
            rows = max(c.max_num_batched_tokens, c.cuda_graph_max_bs, c.max_num_seqs)
            self.symm = SymmetricWorkspace(self.tp, rows=rows, hidden=runner.model.hidden_size,
                                           sample_rows=max(c.cuda_graph_max_bs, c.max_num_seqs))
        elif self.backend == "fused":
            self.backend = "nccl"  # CPU / gloo: no peer memory

    # ------------------------------------------------------------ reductions
    def input_buffer(self, T: int):
        """Where the row-parallel GEMM should write its partial sums (None: anywhere)."""
        if self.symm is not None and T <= self.symm.rows:
            return self.symm.input_buffer(T)
        return None

    def begin_forward(self) -> None:
        if self.symm is not None:
            self.symm.begin_forward()

    def allreduce_add_rmsnorm(self, h, residual, w, eps, final: bool = False):
        """``final``: the last reduction of a forward (the final norm before the lm_head)."""
        if self.symm is not None and h.shape[0] <= self.symm.rows:
            return self.symm.allreduce_add_rmsnorm(h, residual, w, eps, self.ops, final=final)
        dist.all_reduce(h, op=dist.ReduceOp.SUM, group=self.tp.group)
        return self.ops.add_rmsnorm(h, residual, w, eps)

    # ----------------------------------------- GEMM -> reduce-scatter (decode steps)
    def rs_ok(self, T: int, k: int) -> bool:
        """The row-parallel GEMM of a T-token step with inner size k can store its rows at their
        owners (fused backend, decode-sized step, K a multiple of the GEMM's 64-wide k-block)."""
        return self.symm is not None and self.rs_enabled and k % 64 == 0 and self.symm.rs_ok(T)

    def linear_rs_norm(self, x, w, w_norm, eps):
        """rmsnorm(allreduce(x @ w^T) + residual) with the reduce-scatter in the GEMM epilogue:
        the GEMM stores each output row at the rank that owns it, the owner sums the partials,
        adds its residual rows, normalises and all-gathers.  Returns (normed rows, residual)."""
        self.symm.linear_rs(x, w, self.ops)
        return self.symm.rs_add_rmsnorm(x.shape[0], w_norm, eps, self.ops)

    def all_reduce(self, x):
        dist.all_reduce(x, op=dist.ReduceOp.SUM, group=self.tp.group)
        return x

    # ------------------------------------------------------------- sampling
    def vocab_parallel_sample(self, logits, temps, topp, model, runner):
        """Tokens of every row sampled over the whole vocabulary from this rank's shard.

        Fused backend: one kernel per step; the per-row partials (maxima, top-p mass histograms,
        (score, token) pairs) cross the ranks by peer stores into the symmetric buffer, so the
        decode graph holds no NCCL call and no eager op.  NCCL backend (the baseline): the
        (score, token) pairs are all-gathered, or for top-p the whole logits."""
        n = self.tp.size
        use_top_p = getattr(runner, "_use_top_p", False)
        if self.symm is not None and logits.shape[0] <= self.symm.sample_cap:
            return self.symm.sample_rows(logits, temps, topp if use_top_p else None, runner._step_tensor(),
                                         model.vocab_start, self.ops)
        if runner.is_cuda and not use_top_p:
            val, tok = self.ops.sample_partial(logits, temps, runner._step_tensor(), model.vocab_start)
            pair = torch.stack([val, tok.float()], dim=1)  # token ids < 2^24 are exact in fp32
            out = torch.empty(n, *pair.shape, dtype=pair.dtype, device=pair.device)
            dist.all_gather_into_tensor(out, pair.contiguous(), group=self.tp.group)
            best = out[:, :, 0].argmax(dim=0)
            return out[best, torch.arange(pair.shape[0], device=pair.device), 1].to(torch.int32)
        # top-p on the NCCL baseline (or CPU): gather the full logits; every rank samples identically
        parts = [torch.empty_like(logits) for _ in range(n)]
        dist.all_gather(parts, logits.contiguous(), group=self.tp.group)
        full = torch.cat(parts, dim=1)[:, :model.vocab_size]
        return self.ops.sample(full, temps, topp, step=runner._step_tensor(), generator=runner._gen,
                               use_top_p=True, batch_greedy_compat=runner.config.batch_greedy_compat)

    def close(self):
        if self.symm is not None:
            self.symm.close()
            self.symm = None
