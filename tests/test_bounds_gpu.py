"""Index checks of the kernels that scatter or gather by host-supplied indices.

A KV slot beyond the pool, or a gathered norm row beyond the input, is recorded as an error
code and skipped: the valid entries of the same launch are processed normally and the bad one
touches no memory (so a bad index never faults the GPU)."""
import pytest
import torch

from nanovllm_self_b200.ops import torch_ref as R

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    from nanovllm_self_b200.ops.cuda_ops import CudaOps
    o = CudaOps()
    assert int(o.C.BOUNDS_CHECK) == 1
    o.C.bounds_error(True)
    return o


def test_kv_slot_beyond_pool_is_reported_and_skipped(ops):
    nq, nkv, T, nb, bs = 4, 2, 6, 3, 16
    g = torch.Generator(device=DEV).manual_seed(0)
    qkv = torch.randn(T, (nq + 2 * nkv) * 128, device=DEV, generator=g).bfloat16()
    kc = torch.zeros(nb, nkv, bs, 128, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.tensor([0, 5, nb * bs + 7, 17, -1, nb * bs], device=DEV, dtype=torch.int32)
    pos = torch.arange(T, device=DEV, dtype=torch.int32)
    cs = R.rope_cos_sin(128, 64, 1e6, device=DEV)
    w = torch.ones(128, device=DEV, dtype=torch.bfloat16)
    ops.qkv_post(qkv, w, w, 1e-6, pos, cs, kc, vc, slots, None, None, nq, nkv, 128)
    torch.cuda.synchronize()
    assert ops.C.bounds_error(True) == 402
    written = (kc.view(-1, 128).abs().sum(1) > 0).nonzero().flatten().tolist()
    # pool rows are (block, head, offset): the three valid slots, both KV heads, are written
    expect = sorted(((s // bs) * nkv + h) * bs + s % bs for s in (0, 5, 17) for h in range(nkv))
    assert written == expect


def test_gathered_norm_row_out_of_range_is_reported_and_skipped(ops):
    x = torch.randn(5, 256, device=DEV).bfloat16()
    r = torch.randn_like(x)
    w = torch.ones(256, device=DEV, dtype=torch.bfloat16)
    rows = torch.tensor([4, 9, 0], device=DEV, dtype=torch.int32)
    out, res = ops.add_rmsnorm_rows(x, r, w, 1e-6, rows)
    torch.cuda.synchronize()
    assert ops.C.bounds_error(True) == 401
    ref, _ = ops.add_rmsnorm_rows(x, r, w, 1e-6, torch.tensor([4, 0, 0], device=DEV, dtype=torch.int32))
    assert torch.equal(out[0], ref[0]) and torch.equal(out[2], ref[2])
    assert ops.C.bounds_error(True) == 0
