"""The allocation-free decode attention entry point, called through its exported C symbol.

``nvb_attn_decode_noalloc`` serves callers that cannot allocate device memory (for
example code running inside a captured graph with a frozen memory pool, or a host
engine that owns every allocation): it keeps its split-KV scratch in a fixed array
inside the library instead of asking for memory.  This test loads the symbol with
ctypes and checks that two consecutive calls agree with the regular entry point,
which is given torch-allocated scratch.  The file is named so pytest collects it last.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _symbol():
    import nanovllm_self_b200._C as ext
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.nvb_attn_decode_noalloc
    fn.restype = ctypes.c_int
    p, i = ctypes.c_void_p, ctypes.c_int
    fn.argtypes = [p, p, p, p, p, p, i, p, p, p, i, i, i, i, i, i, i, i, ctypes.c_float, p]
    rows = lib.nvb_attn_decode_noalloc_max_rows
    rows.restype = ctypes.c_int
    return ext, fn, rows()


def _case(seed, B, nq, nkv, bs, ctx):
    g = torch.Generator(device=DEV).manual_seed(seed)
    nbps = (ctx + bs - 1) // bs
    nb = B * nbps + 3
    kc = torch.randn(nb, nkv, bs, 128, device=DEV, generator=g).bfloat16()
    vc = torch.randn(nb, nkv, bs, 128, device=DEV, generator=g).bfloat16()
    perm = torch.randperm(nb, device=DEV, generator=g)[:B * nbps].to(torch.int32)
    bt = perm.view(B, nbps).contiguous()
    q = torch.randn(B, nq * 128, device=DEV, generator=g).bfloat16()
    cu = torch.arange(B + 1, device=DEV, dtype=torch.int32)
    lens = torch.randint(1, ctx + 1, (B,), device=DEV, generator=g).to(torch.int32)
    return q, kc, vc, bt, cu, lens


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_matches_regular_entry_point_on_two_calls():
    ext, fn, max_rows = _symbol()
    nq, nkv, bs, splits = 32, 8, 16, 4
    scale = 1.0 / math.sqrt(128)
    for call, (seed, B, ctx) in enumerate([(1, 6, 1500), (2, 9, 700)]):
        assert B * nq * splits <= max_rows
        q, kc, vc, bt, cu, lens = _case(seed, B, nq, nkv, bs, ctx)
        ref = torch.empty_like(q)
        part_o = torch.empty(B * nq * splits * 128, device=DEV)
        part_lse = torch.empty(B * nq * splits, device=DEV)
        ext.attn_decode(q, kc, vc, None, None, bt, cu, lens, ref, part_o, part_lse, nq, nkv, splits, 0, B, scale)
        out = torch.full_like(q, float("nan"))
        stream = torch.cuda.current_stream().cuda_stream
        rc = fn(_ptr(q), _ptr(kc), _ptr(vc), None, None, _ptr(bt), bt.shape[1], _ptr(cu), _ptr(lens), _ptr(out),
                B, nq, nkv, 128, bs, kc.shape[0], 0, splits, ctypes.c_float(scale), ctypes.c_void_p(stream))
        assert rc == 0, f"call {call}: cuda error {rc}"
        torch.cuda.synchronize()
        assert not torch.isnan(out.float()).any()
        err = (out.float() - ref.float()).abs()
        tol = 0.02 + 0.03 * ref.float().abs()
        assert (err > tol).float().mean().item() < 1e-3, f"call {call}: max err {err.max().item()}"


def test_noalloc_rejects_oversized_requests():
    ext, fn, max_rows = _symbol()
    q = torch.zeros(1, 128, device=DEV, dtype=torch.bfloat16)
    too_many_splits = max_rows + 1
    rc = fn(_ptr(q), _ptr(q), _ptr(q), None, None, _ptr(q), 1, _ptr(q), _ptr(q), _ptr(q),
            1, 1, 1, 128, 16, 1, 0, too_many_splits, ctypes.c_float(1.0), None)
    assert rc != 0
