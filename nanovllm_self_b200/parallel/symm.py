"""Symmetric device buffers shared by the TP ranks through CUDA IPC.

Each rank ``cudaMalloc``s one buffer (via the extension, outside torch's caching
allocator), exports its IPC handle, gathers every peer's handle over the process group
and opens them, so every rank holds a pointer to every rank's buffer.  The buffer is
laid out as ``IN | RES | OUT | FLAGS`` (see ``csrc/comm.cu``).  The fused
``allreduce_add_rmsnorm`` kernel reads the peers' IN rows and writes every rank's RES
and OUT rows over NVLink.
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
    CTAS = 32

    def __init__(self, tp, rows: int, hidden: int):
        self.C = load()
        self.tp = tp
        self.rows = rows
        self.hidden = hidden
        row_bytes = rows * hidden * 2
        self.in_off = 0
        self.res_off = row_bytes
        self.out_off = 2 * row_bytes
        self.flag_off = 3 * row_bytes
        self.nbytes = 3 * row_bytes + int(self.C.COMM_FLAG_BYTES)
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
        view = raw[:3 * row_bytes].view(torch.bfloat16).view(3, rows, hidden)
        self.IN, self.RES, self.OUT = view[0], view[1], view[2]
        self.epochs = torch.zeros(self.C.COMM_MAX_CTAS, dtype=torch.int32, device=tp.device)
        dist.barrier(group=tp.group)

    def input_buffer(self, T: int) -> torch.Tensor:
        return self.IN[:T]

    def allreduce_add_rmsnorm(self, h, residual, w, eps, ops=None):
        T = h.shape[0]
        if T > self.rows:
            raise ValueError(f"{T} rows exceed the symmetric workspace ({self.rows})")
        inv = self.IN[:T]
        if h.data_ptr() != inv.data_ptr():
            inv.copy_(h)
        res = self.RES[:T]
        has_res = residual is not None
        if has_res and residual.data_ptr() != res.data_ptr():
            res.copy_(residual)
        self.C.allreduce_add_rmsnorm(self.bases, self.in_off, self.res_off, self.out_off, self.flag_off,
                                     self.epochs, w, self.tp.rank, T, self.hidden, has_res, float(eps), self.CTAS)
        if ops is not None and hasattr(ops, "launches"):
            ops.launches += 1
        return self.OUT[:T], res

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
