"""Symmetric device buffers shared by the TP ranks through CUDA IPC.

Each rank ``cudaMalloc``s one buffer (via the extension, outside torch's caching
allocator), exports its IPC handle, gathers every peer's handle over the process group
and opens them, so every rank holds a pointer to every rank's buffer.  The buffer is
laid out as ``IN | IN0 IN1 IN2 | RES | OUT | RS | FLAGS`` (see ``csrc/comm.cu``).  The fused
``allreduce_add_rmsnorm`` kernel reads the peers' IN rows and writes every rank's RES
and OUT rows over NVLink.

Decode-sized steps (at most ``COMM_RS_MAX_ROWS`` tokens) take the GEMM -> reduce-scatter
path instead: the row-parallel GEMM stores each output row straight into the RS area of
the rank that owns it (``linear_rs``), and one kernel on the owner sums the partials, adds
the residual, normalises and all-gathers the rows into every rank's OUT
(``rs_add_rmsnorm``).  Only the owner keeps the residual of its rows there.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import load


class _DevPtr:
    """Minimal ``__cuda_array_interface__`` wrapper to view raw device memory as a tensor."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


class SymmetricWorkspace:

    # one-shot while the bytes each rank pulls from its peers, (world - 1) * T * H * 2,
    # stay below this; beyond it the two-shot kernel moves 2 (world - 1) / world of that
    ONESHOT_PEER_BYTES = 4 << 20

    def __init__(self, tp, rows: int, hidden: int, oneshot_rows: int | None = None, timeout_s: float = 10.0,
                 sample_rows: int = 0):
        self.C = load()
        # bound of every peer wait inside the kernels; on expiry they record an error word
        # (``error()``) and return instead of waiting for ever
        self.timeout_ns = int(timeout_s * 1e9)
        self.tp = tp
        self.rows = rows
        self.hidden = hidden
        if oneshot_rows is None:
            oneshot_rows = max(1, min(512, self.ONESHOT_PEER_BYTES // (max(1, tp.size - 1) * hidden * 2)))
        self.oneshot_rows = oneshot_rows
        # every CTA of a call must be resident at once (the per-rank barrier releases them)
        self.max_ctas = min(int(self.C.COMM_MAX_CTAS),
                            torch.cuda.get_device_properties(tp.device).multi_processor_count)
        row_bytes = rows * hidden * 2
        small = min(rows, oneshot_rows) * hidden * 2
        self.rs_max_rows = int(self.C.COMM_RS_MAX_ROWS)
        rs_bytes = tp.size * self.rs_max_rows * hidden * 2
        # IN (two-shot) | IN0 IN1 IN2 (one-shot rotation) | RES | OUT | RS (reduce-scatter) | FLAGS
        self.in_off = 0
        self.in1_off = [row_bytes, row_bytes + small, row_bytes + 2 * small]
        self.res_off = row_bytes + 3 * small
        self.out_off = 2 * row_bytes + 3 * small
        self.rs_off = 3 * row_bytes + 3 * small
        # sampler exchange (vocab-parallel sampling): SX floats, SF flag words
        self.sample_cap = int(sample_rows)
        sx = int(self.C.sample_x_floats(tp.size, self.sample_cap)) * 4 if self.sample_cap else 0
        sf = int(self.C.sample_f_words(tp.size, self.sample_cap)) * 4 if self.sample_cap else 0
        self.sx_off = self.rs_off + rs_bytes
        self.sf_off = self.sx_off + ((sx + 255) // 256) * 256
        self.flag_off = self.sf_off + ((sf + 255) // 256) * 256
        self.nbytes = self.flag_off + int(self.C.COMM_FLAG_BYTES)
        torch.cuda.set_device(tp.device)
        self.base, handle = self.C.symm_alloc(self.nbytes)
        handles = [None] * tp.size
        dist.all_gather_object(handles, handle, group=tp.group)
        self.bases = []
        self._opened = []
        for p, h in enumerate(handles):
            if p == tp.rank:
                self.bases.append(self.base)
            else:
                ptr = self.C.symm_open(h)
                self._opened.append(ptr)
                self.bases.append(ptr)
        raw = torch.as_tensor(_DevPtr(self.base, self.nbytes), device=tp.device)
        self._raw = raw

        def view(off, n):
            return raw[off:off + n * hidden * 2].view(torch.bfloat16).view(n, hidden)
        self.IN = view(self.in_off, rows)
        self.IN1 = [view(o, min(rows, oneshot_rows)) for o in self.in1_off]
        self.RES = view(self.res_off, rows)
        self.OUT = view(self.out_off, rows)
        # One-shot IN buffers: the layers' reductions of a forward alternate between buffers 0
        # and 1 (reset at every forward), the forward's last reduction (the final norm) uses
        # buffer 2.  So two consecutive reductions never share a buffer, inside a forward or
        # across the boundary of two forwards (CUDA-graph replays repeat the same sequence):
        # a rank then refills a buffer only after a barrier that every peer passed after its
        # reads of that buffer (the protocol model in the tests checks this).
        self._k = 0
        dist.barrier(group=tp.group)

    def _oneshot(self, T: int) -> bool:
        return T <= self.oneshot_rows

    def begin_forward(self) -> None:
        self._k = 0

    def _slot(self, final: bool) -> int:
        return 2 if final else self._k % 2

    def input_buffer(self, T: int, final: bool = False) -> torch.Tensor:
        """Where the next reduction's input should be written (the GEMM writes straight here)."""
        if self._oneshot(T):
            return self.IN1[self._slot(final)][:T]
        return self.IN[:T]

    def allreduce_add_rmsnorm(self, h, residual, w, eps, ops=None, final: bool = False):
        T = h.shape[0]
        if T > self.rows:
            raise ValueError(f"{T} rows exceed the symmetric workspace ({self.rows})")
        one = self._oneshot(T)
        inv = self.input_buffer(T, final)
        in_off = self.in1_off[self._slot(final)] if one else self.in_off
        if h.data_ptr() != inv.data_ptr():
            inv.copy_(h)
        res = self.RES[:T]
        has_res = residual is not None
        if has_res and residual.data_ptr() != res.data_ptr():
            res.copy_(residual)
        if one:
            ctas = max(1, min(self.max_ctas, T))
        else:
            ctas = max(1, min(self.max_ctas, (T + self.tp.size - 1) // self.tp.size))
        self.C.allreduce_add_rmsnorm(self.bases, in_off, self.res_off, self.out_off, self.flag_off,
                                     w, self.tp.rank, T, self.hidden, has_res, float(eps), ctas, one, self.timeout_ns)
        if one and not final:
            self._k += 1
        if ops is not None and hasattr(ops, "launches"):
            ops.launches += 1
        return self.OUT[:T], res

    # ------------------------------------------------ GEMM -> reduce-scatter path
    def rs_ok(self, T: int) -> bool:
        """Whether a step of T tokens can take the GEMM -> reduce-scatter path."""
        return 0 < T <= min(self.rs_max_rows, self.rows)

    def rs_rows(self, T: int) -> int:
        return (T + self.tp.size - 1) // self.tp.size

    def linear_rs(self, x, w, ops=None):
        """Row-parallel GEMM x @ w^T whose output rows are stored at their owner ranks."""
        T = x.shape[0]
        plan = self.C.linear_rs(x, w, self.bases, self.rs_off, self.flag_off, self.tp.rank, self.rs_rows(T),
                                self.IN[:T])
        if ops is not None and hasattr(ops, "launches"):
            ops.launches += 1
        return plan

    def rs_add_rmsnorm(self, T: int, w, eps, ops=None):
        """Owner-side sum + residual + RMSNorm + all-gather of the rows ``linear_rs`` stored.

        Returns (OUT[:T], RES[:T]): every rank holds all normalised rows; the residual rows
        are current only on their owner (they are only ever read there).
        """
        rr = self.rs_rows(T)
        ctas = max(1, min(self.max_ctas, rr))
        self.C.rs_add_rmsnorm_ag(self.bases, self.rs_off, self.res_off, self.out_off, self.flag_off, w,
                                 self.tp.rank, T, rr, self.hidden, True, float(eps), ctas, self.timeout_ns)
        if ops is not None and hasattr(ops, "launches"):
            ops.launches += 1
        return self.OUT[:T], self.RES[:T]

    # ------------------------------------------------------- vocab-parallel sampling
    def sample_rows(self, logits, temps, top_p, step, col_offset: int, ops=None):
        """Sample every row over the whole vocabulary from this rank's shard of the logits: the
        kernel combines the shards with the other ranks through the symmetric buffer (per-row
        maxima, top-p mass histograms and (score, token) pairs, by NVLink peer stores).  Every
        rank returns the same tokens."""
        rows = logits.shape[0]
        if rows > self.sample_cap:
            raise ValueError(f"{rows} rows exceed the sampler exchange capacity ({self.sample_cap})")
        tok = torch.empty(rows, dtype=torch.int32, device=logits.device)
        xb = [b + self.sx_off for b in self.bases]
        fb = [b + self.sf_off for b in self.bases]
        self.C.sample_rows(logits, int(col_offset), temps, top_p, step, tok, None, xb, fb, self.tp.rank,
                           self.sample_cap, self.timeout_ns)
        if ops is not None and hasattr(ops, "launches"):
            ops.launches += 1
        return tok

    def error(self, reset: bool = False) -> int:
        return int(self.C.comm_error(reset))

    def close(self):
        torch.cuda.synchronize(self.tp.device)
        for p in self._opened:
            try:
                self.C.symm_close(p)
            except RuntimeError:
                pass
        self._opened = []
        if self.base:
            self.C.symm_free(self.base)
            self.base = 0
