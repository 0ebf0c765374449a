"""The allocation-free decode attention entry point, called through its exported C symbol.

``nvb_attn_decode_noalloc`` serves callers that cannot allocate device memory (for
example code running inside a captured graph with a frozen memory pool, or a host
engine that owns every allocation): it keeps its split-KV scratch in a fixed array
inside the library instead of asking for memory.  These tests load the symbol with
ctypes (its C declaration is ``csrc/attn_decode_noalloc.h``) and check that two
consecutive calls agree with the regular entry point, which is given torch-allocated
scratch, over bf16 and fp8 KV, block sizes 16 and 256 and one or several splits.
The file is named so pytest collects it last.
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
    rows.argtypes = []
    return ext, fn, rows()


def _case(seed, B, nq, nkv, bs, ctx, fp8, min_len=1):
    g = torch.Generator(device=DEV).manual_seed(seed)
    nbps = (ctx + bs - 1) // bs
    nb = B * nbps + 3
    kc = torch.randn(nb, nkv, bs, 128, device=DEV, generator=g)
    vc = torch.randn(nb, nkv, bs, 128, device=DEV, generator=g)
    ks = vs = None
    if fp8:
        ks = torch.rand(nb, nkv, device=DEV, generator=g) * 0.05 + 0.01
        vs = torch.rand(nb, nkv, device=DEV, generator=g) * 0.05 + 0.01
        kc, vc = kc.to(torch.float8_e4m3fn), vc.to(torch.float8_e4m3fn)
    else:
        kc, vc = kc.bfloat16(), vc.bfloat16()
    perm = torch.randperm(nb, device=DEV, generator=g)[:B * nbps].to(torch.int32)
    bt = perm.view(B, nbps).contiguous()
    q = torch.randn(B, nq * 128, device=DEV, generator=g).bfloat16()
    cu = torch.arange(B + 1, device=DEV, dtype=torch.int32)
    lens = torch.randint(min_len, ctx + 1, (B,), device=DEV, generator=g).to(torch.int32)
    return q, kc, vc, ks, vs, bt, cu, lens


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _poison_scratch(ext, fn, max_rows):
    """Fill every row of the library's scratch with NaN partial outputs.

    A call whose V cache is all NaN writes NaN into every partial-output row it uses; with
    num_seqs * nq * splits equal to the maximum, that is the whole array.
    """
    nq, nkv, bs, splits = 8, 8, 16, 64
    B = max_rows // (nq * splits)
    ctx = 64 * splits
    q, kc, vc, _, _, bt, cu, _ = _case(7, B, nq, nkv, bs, ctx, False)
    vc.fill_(float("nan"))
    lens = torch.full((B,), ctx, device=DEV, dtype=torch.int32)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(_ptr(q), _ptr(kc), _ptr(vc), None, None, _ptr(bt), bt.shape[1], _ptr(cu), _ptr(lens), _ptr(out),
            B, nq, nkv, 128, bs, kc.shape[0], 0, splits, ctypes.c_float(0.1), ctypes.c_void_p(stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.isnan(out.float()).all()


@pytest.mark.parametrize("fp8,bs,splits", [(False, 16, 4), (True, 16, 4), (False, 256, 3), (True, 256, 1),
                                           (False, 16, 1)])
def test_noalloc_matches_regular_entry_point_on_two_calls(fp8, bs, splits):
    ext, fn, max_rows = _symbol()
    nq, nkv = 32, 8
    scale = 1.0 / math.sqrt(128)
    for call, (seed, B, ctx) in enumerate([(1, 6, 1500), (2, 9, 700)]):
        assert B * nq * splits <= max_rows
        q, kc, vc, ks, vs, bt, cu, lens = _case(seed, B, nq, nkv, bs, ctx, fp8)
        ref = torch.empty_like(q)
        part_o = torch.empty(B * nq * splits * 128, device=DEV)
        part_lse = torch.empty(B * nq * splits, device=DEV)
        ext.attn_decode(q, kc, vc, ks, vs, bt, cu, lens, ref, part_o, part_lse, nq, nkv, splits, 0, B, scale)
        out = torch.full_like(q, float("nan"))
        stream = torch.cuda.current_stream().cuda_stream
        rc = fn(_ptr(q), _ptr(kc), _ptr(vc), _ptr(ks), _ptr(vs), _ptr(bt), bt.shape[1], _ptr(cu), _ptr(lens),
                _ptr(out), B, nq, nkv, 128, bs, kc.shape[0], int(fp8), splits, ctypes.c_float(scale),
                ctypes.c_void_p(stream))
        assert rc == 0, f"call {call}: cuda error {rc}"
        torch.cuda.synchronize()
        assert not torch.isnan(out.float()).any()
        err = (out.float() - ref.float()).abs()
        tol = 0.02 + 0.03 * ref.float().abs()
        assert (err > tol).float().mean().item() < 1e-3, f"call {call}: max err {err.max().item()}"


def test_noalloc_ignores_stale_nan_scratch_for_empty_splits():
    """Contexts shorter than `splits` key tiles leave splits empty; stale NaN rows must not leak."""
    ext, fn, max_rows = _symbol()
    _poison_scratch(ext, fn, max_rows)
    nq, nkv, bs, splits = 32, 8, 16, 8
    scale = 1.0 / math.sqrt(128)
    for call in range(2):
        q, kc, vc, _, _, bt, cu, _ = _case(11 + call, 5, nq, nkv, bs, 100, False)
        lens = torch.tensor([1, 3, 64, 65, 100], device=DEV, dtype=torch.int32)  # 1-2 key tiles of 64
        ref = torch.empty_like(q)
        part_o = torch.full((5 * nq * splits * 128,), float("nan"), device=DEV)
        part_lse = torch.empty(5 * nq * splits, device=DEV)
        ext.attn_decode(q, kc, vc, None, None, bt, cu, lens, ref, part_o, part_lse, nq, nkv, splits, 0, 5, scale)
        out = torch.full_like(q, float("nan"))
        stream = torch.cuda.current_stream().cuda_stream
        rc = fn(_ptr(q), _ptr(kc), _ptr(vc), None, None, _ptr(bt), bt.shape[1], _ptr(cu), _ptr(lens), _ptr(out),
                5, nq, nkv, 128, bs, kc.shape[0], 0, splits, ctypes.c_float(scale), ctypes.c_void_p(stream))
        assert rc == 0
        torch.cuda.synchronize()
        assert not torch.isnan(ref.float()).any(), "regular entry point read a stale NaN row"
        assert not torch.isnan(out.float()).any(), "allocation-free entry point read a stale NaN row"
        assert torch.allclose(out.float(), ref.float(), atol=2e-2, rtol=3e-2)


def test_noalloc_rejects_bad_arguments():
    ext, fn, max_rows = _symbol()
    q = torch.zeros(1, 128, device=DEV, dtype=torch.bfloat16)
    i32 = torch.zeros(2, device=DEV, dtype=torch.int32)

    def call(nq=1, nkv=1, bs=16, nb=1, splits=1, head_dim=128, width=1, fp8=0):
        return fn(_ptr(q), _ptr(q), _ptr(q), None, None, _ptr(i32), width, _ptr(i32), _ptr(i32), _ptr(q),
                  1, nq, nkv, head_dim, bs, nb, fp8, splits, ctypes.c_float(1.0), None)

    assert call(splits=max_rows + 1) != 0
    assert call(nkv=0) != 0
    assert call(nq=0) != 0
    assert call(nq=3, nkv=2) != 0
    assert call(bs=0) != 0
    assert call(bs=24) != 0
    assert call(nb=0) != 0
    assert call(head_dim=64) != 0
    assert call(fp8=1) != 0  # fp8 KV without scales
