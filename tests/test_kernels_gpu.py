"""Numerics of every sm_100a kernel against the plain-PyTorch fp32 reference of the same op."""
import math

import pytest
import torch

from nanovllm_self_b200.ops import torch_ref as R

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    from nanovllm_self_b200.ops.cuda_ops import CudaOps
    return CudaOps()


def _close(a, b, atol, rtol=0.02):
    a, b = a.float(), b.float()
    err = (a - b).abs()
    tol = atol + rtol * b.abs()
    bad = (err > tol).float().mean().item()
    assert bad < 1e-3, f"{bad*100:.3f}% elements out of tolerance, max err {err.max().item():.4g}"


@pytest.mark.parametrize("rows,H", [(1, 1024), (7, 4096), (300, 5120), (33, 256)])
@pytest.mark.parametrize("with_res", [False, True])
def test_add_rmsnorm(ops, rows, H, with_res):
    g = torch.Generator(device=DEV).manual_seed(rows + H)
    x = torch.randn(rows, H, device=DEV, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(H, device=DEV, generator=g)).bfloat16()
    res = torch.randn(rows, H, device=DEV, generator=g).bfloat16() if with_res else None
    ref_out, ref_res = R.add_rmsnorm(x.float(), None if res is None else res.float(), w.float(), 1e-6)
    out, r = ops.add_rmsnorm(x, None if res is None else res.clone(), w, 1e-6)
    _close(out, ref_out, 0.02)
    _close(r, ref_res, 0.02)


def test_add_rmsnorm_rows(ops):
    h = torch.randn(50, 1024, device=DEV).bfloat16()
    res = torch.randn(50, 1024, device=DEV).bfloat16()
    w = torch.ones(1024, device=DEV).bfloat16()
    rows = torch.tensor([3, 49, 0, 17], device=DEV, dtype=torch.int32)
    out, _ = ops.add_rmsnorm_rows(h, res, w, 1e-6, rows)
    ref, _ = R.add_rmsnorm(h[rows.long()].float(), res[rows.long()].float(), w.float(), 1e-6)
    _close(out, ref, 0.02)


@pytest.mark.parametrize("T,I", [(1, 3072), (129, 12288), (5, 1536)])
def test_silu_mul(ops, T, I):
    x = torch.randn(T, 2 * I, device=DEV).bfloat16()
    _close(ops.silu_mul(x), R.silu_mul(x.float()), 0.01)


def test_embedding_shard(ops):
    w = torch.randn(100, 256, device=DEV).bfloat16()
    ids = torch.tensor([0, 150, 175, 249, 250, 3], device=DEV, dtype=torch.int32)
    out = ops.embedding(ids, w, 150)
    ref = R.embedding(ids, w, 150)
    assert torch.equal(out, ref)


def _kv_setup(nb, nkv, bs, dtype, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    kc = torch.zeros(nb, nkv, bs, 128, device=DEV, dtype=dtype)
    vc = torch.zeros_like(kc)
    ks = vs = None
    if dtype == torch.float8_e4m3fn:
        ks = torch.ones(nb, nkv, device=DEV)
        vs = torch.ones(nb, nkv, device=DEV)
    return kc, vc, ks, vs, g


@pytest.mark.parametrize("kv_dtype", [torch.bfloat16, torch.float8_e4m3fn])
@pytest.mark.parametrize("bs", [16, 256])
@pytest.mark.parametrize("nq,nkv", [(8, 2), (32, 8), (5, 1)])
def test_qkv_post(ops, kv_dtype, bs, nq, nkv):
    # (32, 8): Qwen3-8B heads, a warp's 16 heads straddle the K / V boundary; (5, 1): the two
    # halves of a warp take a query head and a key head in the same pass
    T = 40
    nb = 16
    kc, vc, ks, vs, g = _kv_setup(nb, nkv, bs, kv_dtype)
    qkv = torch.randn(T, (nq + 2 * nkv) * 128, device=DEV, generator=g).bfloat16()
    qn = (1 + 0.1 * torch.randn(128, device=DEV, generator=g)).bfloat16()
    kn = (1 + 0.1 * torch.randn(128, device=DEV, generator=g)).bfloat16()
    pos = torch.arange(5, 5 + T, device=DEV, dtype=torch.int32)
    cs = R.rope_cos_sin(128, 4096, 1e6, device=DEV)
    # tokens 5.. of a sequence whose block table is [3, 7, 1, ...]; slot -1 for the last token
    table = torch.tensor([3, 7, 1, 9, 11, 2, 4, 5], device=DEV)
    p = pos.long()
    slots = (table[p // bs] * bs + p % bs).to(torch.int32)
    slots[-1] = -1
    q = ops.qkv_post(qkv, qn, kn, 1e-6, pos, cs, kc, vc, slots, ks, vs, nq, nkv, 128)
    kc2, vc2 = torch.zeros_like(kc, dtype=torch.float32), torch.zeros_like(vc, dtype=torch.float32)
    ks2 = vs2 = None
    if kv_dtype == torch.float8_e4m3fn:
        kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
        ks2, vs2 = torch.ones_like(ks), torch.ones_like(vs)
    qf = qkv.float()
    qr = R.apply_rope(R.rmsnorm(qf[:, :nq * 128].reshape(T, nq, 128), qn.float(), 1e-6), pos, cs)
    kr = R.apply_rope(R.rmsnorm(qf[:, nq * 128:(nq + nkv) * 128].reshape(T, nkv, 128), kn.float(), 1e-6), pos, cs)
    vr = qf[:, (nq + nkv) * 128:].reshape(T, nkv, 128)
    R.store_kv(kr, vr, kc2, vc2, slots, ks2, vs2)
    _close(q.view(T, nq, 128), qr, 0.03)
    if kv_dtype == torch.float8_e4m3fn:
        _close(kc.float() * ks[:, :, None, None], kc2.float() * ks2[:, :, None, None], 0.05, 0.08)
        _close(vc.float() * vs[:, :, None, None], vc2.float() * vs2[:, :, None, None], 0.05, 0.08)
        _close(ks, ks2, 1e-3)
    else:
        _close(kc, kc2, 0.03)
        _close(vc, vc2, 0.03)


@pytest.mark.parametrize("kv_dtype", [torch.bfloat16, torch.float8_e4m3fn])
@pytest.mark.parametrize("nq,nkv", [(32, 8), (8, 2), (4, 1)])
def test_qkv_post_many_chunks(ops, kv_dtype, nq, nkv):
    # enough tokens that every CTA of the persistent kernel refills its stage ring several times,
    # and a count that is not a multiple of the tokens per stage (the last stage is partial)
    T, bs = 9001, 16
    nb = (T + bs - 1) // bs + 3
    kc, vc, ks, vs, g = _kv_setup(nb, nkv, bs, kv_dtype, seed=2)
    qkv = torch.randn(T, (nq + 2 * nkv) * 128, device=DEV, generator=g).bfloat16()
    qn = (1 + 0.1 * torch.randn(128, device=DEV, generator=g)).bfloat16()
    kn = (1 + 0.1 * torch.randn(128, device=DEV, generator=g)).bfloat16()
    pos = torch.arange(T, device=DEV, dtype=torch.int32)
    cs = R.rope_cos_sin(128, 16384, 1e6, device=DEV)
    table = torch.randperm(nb, generator=torch.Generator().manual_seed(3)).to(DEV)
    p = pos.long()
    slots = (table[p // bs] * bs + p % bs).to(torch.int32)
    q = ops.qkv_post(qkv, qn, kn, 1e-6, pos, cs, kc, vc, slots, ks, vs, nq, nkv, 128)
    kc2, vc2 = torch.zeros_like(kc, dtype=torch.float32), torch.zeros_like(vc, dtype=torch.float32)
    ks2 = vs2 = None
    if kv_dtype == torch.float8_e4m3fn:
        kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
        ks2, vs2 = torch.ones_like(ks), torch.ones_like(vs)
    qf = qkv.float()
    qr = R.apply_rope(R.rmsnorm(qf[:, :nq * 128].reshape(T, nq, 128), qn.float(), 1e-6), pos, cs)
    kr = R.apply_rope(R.rmsnorm(qf[:, nq * 128:(nq + nkv) * 128].reshape(T, nkv, 128), kn.float(), 1e-6), pos, cs)
    vr = qf[:, (nq + nkv) * 128:].reshape(T, nkv, 128)
    R.store_kv(kr, vr, kc2, vc2, slots, ks2, vs2)
    _close(q.view(T, nq, 128), qr, 0.03)
    if kv_dtype == torch.float8_e4m3fn:
        _close(kc.float() * ks[:, :, None, None], kc2.float() * ks2[:, :, None, None], 0.05, 0.08)
        _close(vc.float() * vs[:, :, None, None], vc2.float() * vs2[:, :, None, None], 0.05, 0.08)
        _close(ks, ks2, 1e-3)
    else:
        _close(kc, kc2, 0.03)
        _close(vc, vc2, 0.03)
    assert ops.C.bounds_error(True) == 0


def _paged_case(q_lens, k_lens, nq, nkv, bs, kv_dtype, seed=1):
    nb = sum((k + bs - 1) // bs for k in k_lens) + 4
    g = torch.Generator(device=DEV).manual_seed(seed)
    kf = torch.randn(nb, nkv, bs, 128, device=DEV, generator=g)
    vf = torch.randn(nb, nkv, bs, 128, device=DEV, generator=g)
    ks = vs = None
    if kv_dtype == torch.float8_e4m3fn:
        ks = (kf.abs().amax(dim=(2, 3)) / 448.0 * 1.5).float()
        vs = (vf.abs().amax(dim=(2, 3)) / 448.0 * 1.5).float()
        kc = (kf / ks[:, :, None, None]).to(kv_dtype)
        vc = (vf / vs[:, :, None, None]).to(kv_dtype)
    else:
        kc, vc = kf.to(kv_dtype), vf.to(kv_dtype)
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(seed)).tolist()
    W = max((k + bs - 1) // bs for k in k_lens)
    tables, o = [], 0
    for k in k_lens:
        n = (k + bs - 1) // bs
        tables.append(perm[o:o + n] + [0] * (W - n))
        o += n
    T = sum(q_lens)
    q = torch.randn(T, nq, 128, device=DEV, generator=g).bfloat16()
    bt = torch.tensor(tables, device=DEV, dtype=torch.int32)
    cu = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), device=DEV, dtype=torch.int32)
    ctx_lens = torch.tensor(k_lens, device=DEV, dtype=torch.int32)
    return q, kc, vc, ks, vs, bt, cu, ctx_lens, tables


class _Ctx:
    pass


@pytest.mark.parametrize("kv_dtype", [torch.bfloat16, torch.float8_e4m3fn])
@pytest.mark.parametrize("nq,nkv", [(16, 8), (32, 8), (4, 1), (64, 8), (16, 1)])
@pytest.mark.parametrize("bs", [16, 256])
def test_attention_decode_and_prefill(ops, kv_dtype, nq, nkv, bs):
    # 3 decode seqs (various ctx incl. long for split-KV) then 3 prefill seqs (prefix offset, chunk)
    q_lens = [1, 1, 1, 37, 130, 64]
    k_lens = [1, 300, 2100, 37, 200, 1000]
    q, kc, vc, ks, vs, bt, cu, cl, tables = _paged_case(q_lens, k_lens, nq, nkv, bs, kv_dtype)
    ctx = _Ctx()
    ctx.num_decode_seqs, ctx.num_seqs = 3, 6
    ctx.block_tables, ctx.cu_seqlens_q, ctx.context_lens = bt, cu, cl
    ctx.max_seqlen_q, ctx.max_seqlen_k = max(q_lens), max(k_lens)
    scale = 1 / math.sqrt(128)
    out = ops.attention(q.view(q.shape[0], -1), kc, vc, ctx, scale, ks, vs).view_as(q)
    ref = R.paged_attention(q.float(), kc, vc, q_lens, k_lens, tables, scale, ks, vs)
    _close(out, ref, 0.02, 0.03)


@pytest.mark.parametrize("nq,nkv,bs", [(32, 8, 256), (16, 8, 16), (64, 8, 256), (8, 8, 32), (16, 1, 256)])
def test_prefill_tcgen05_matches_fp32(ops, nq, nkv, bs):
    """The tcgen05 prefill kernel (bf16 KV): long prompts, prefix offsets, ragged tails."""
    q_lens = [1000, 300, 129, 7, 512]
    k_lens = [1000, 1300, 129, 700, 2100]
    q, kc, vc, ks, vs, bt, cu, cl, tables = _paged_case(q_lens, k_lens, nq, nkv, bs, torch.bfloat16, seed=3)
    ctx = _Ctx()
    ctx.num_decode_seqs, ctx.num_seqs = 0, len(q_lens)
    ctx.block_tables, ctx.cu_seqlens_q, ctx.context_lens = bt, cu, cl
    ctx.max_seqlen_q, ctx.max_seqlen_k = max(q_lens), max(k_lens)
    scale = 1 / math.sqrt(128)
    ops.C.attn_error(True)
    out = ops.attention(q.view(q.shape[0], -1), kc, vc, ctx, scale).view_as(q)
    torch.cuda.synchronize()
    assert ops.C.attn_error(True) == 0
    ref = R.paged_attention(q.float(), kc, vc, q_lens, k_lens, tables, scale)
    _close(out, ref, 0.02, 0.03)
    # same answer as the mma.sync kernel
    ops.prefill_tc = False
    try:
        out2 = ops.attention(q.view(q.shape[0], -1), kc, vc, ctx, scale).view_as(q)
    finally:
        ops.prefill_tc = True
    _close(out, out2, 0.02, 0.03)


def test_sample_greedy_and_temperature(ops):
    torch.manual_seed(0)
    V = 151936
    logits = torch.randn(6, V, device=DEV)
    logits[:, 1234] += 50
    temps = torch.tensor([0, 0, 0.5, 1.0, 0, 2.0], device=DEV)
    step = torch.tensor([7, 3], dtype=torch.int64, device=DEV)
    tok = ops.sample(logits, temps, step=step)
    assert torch.equal(tok[temps <= 0].long(), logits[temps <= 0].argmax(-1))
    assert (tok[temps > 0] == 1234).all()
    # temperature sampling follows softmax(l / T): check a 4-way distribution
    small = torch.log(torch.tensor([[0.1, 0.2, 0.3, 0.4]], device=DEV)).repeat(4096, 1)
    counts = torch.zeros(4)
    for s in range(4):
        step = torch.tensor([11, s], dtype=torch.int64, device=DEV)
        t = ops.sample(small, torch.ones(4096, device=DEV), step=step)
        counts += torch.bincount(t.long().cpu(), minlength=4).float()
    freq = counts / counts.sum()
    assert torch.allclose(freq, torch.tensor([0.1, 0.2, 0.3, 0.4]), atol=0.02), freq


@pytest.mark.parametrize("rows,V,ld", [(256, 151936, 151936), (3, 151936, 151936), (5, 151941, 151944),
                                       (4, 18992, 18992), (2, 1001, 1003)])
def test_sample_bf16_rows(ops, rows, V, ld):
    # bf16 logits: the bulk-copy path (16-byte aligned rows, with a column tail when V % 8 != 0), and
    # rows whose stride breaks the alignment (plain loads); bf16 rows hold many exact ties, and the
    # first maximum must win as in torch.argmax
    g = torch.Generator(device=DEV).manual_seed(rows + V)
    full = torch.randn(rows, ld, device=DEV, generator=g).bfloat16()
    logits = full[:, :V]
    logits[0, V - 1] = 9.0  # the winner in the tail (or the last vector) of row 0
    if rows > 1:
        logits[1, 3] = 9.0
        logits[1, V // 2] = 9.0  # a tie: the first column wins
    temps = torch.zeros(rows, device=DEV)
    step = torch.tensor([5, 1], dtype=torch.int64, device=DEV)
    tok = ops.sample(logits, temps, step=step)
    assert torch.equal(tok.long(), logits.float().argmax(-1))
    # temperature: a dominant column is always drawn; a 4-way distribution follows softmax(l / T)
    hot = logits.clone()
    hot[:, V // 3] = 60.0
    tok = ops.sample(hot, torch.ones(rows, device=DEV), step=step)
    assert bool((tok == V // 3).all())
    small = torch.log(torch.tensor([[0.1, 0.2, 0.3, 0.4]], device=DEV)).repeat(4096, 1).bfloat16()
    counts = torch.zeros(4)
    for s in range(4):
        t = ops.sample(small, torch.ones(4096, device=DEV), step=torch.tensor([13, s], dtype=torch.int64, device=DEV))
        counts += torch.bincount(t.long().cpu(), minlength=4).float()
    freq = counts / counts.sum()
    ref = torch.softmax(small[0].float(), -1).cpu()
    assert torch.allclose(freq, ref, atol=0.02), (freq, ref)
    assert ops.C.sample_error(True) == 0


@pytest.mark.parametrize("m", [1, 7, 64, 256, 300])
@pytest.mark.parametrize("n,col_offset", [(151936, 0), (18992, 37984), (1000, 0)])
def test_lm_head_sample_matches_logits_path(ops, m, n, col_offset):
    """The lm_head GEMM with the sampler in its epilogue draws exactly the tokens of the same GEMM
    writing bf16 logits followed by the sampler kernel (greedy and temperature rows, same noise),
    in both orientations, tile widths and stream-K, and leaves its key scratch zeroed."""
    k = 1024
    g = torch.Generator(device=DEV).manual_seed(m * 7 + n)
    x = torch.randn(m, k, device=DEV, generator=g).bfloat16()
    w = (torch.randn(n, k, device=DEV, generator=g) * 0.05).bfloat16()
    temps = torch.tensor([0.0, 0.7, 0.0, 1.3], device=DEV).repeat((m + 3) // 4)[:m].contiguous()
    step = torch.tensor([3, 5], dtype=torch.int64, device=DEV)
    sc = ops.scratch(DEV)
    plans = [(0, 128, 1), (0, 256, 1), (0, 128, -1)]
    if m <= 256:
        plans.append((1, 0, 1))
    for swap, bn, splits in plans:
        tok = torch.empty(m, dtype=torch.int32, device=DEV)
        ops.C.linear_sample(x, w, sc.sample_keys, temps, step, col_offset, tok, None, sc.gemm, sc.gemm_counters,
                            False, swap, bn, splits)
        logits = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
        ops.C.linear(x, w, logits, sc.gemm, sc.gemm_counters, swap, bn, splits, 0)
        ref = ops.sample(logits, temps, step=step, col_offset=col_offset)
        assert torch.equal(tok, ref), (swap, bn, splits, (tok != ref).nonzero()[:4].tolist())
        assert bool((sc.sample_keys[:m] == 0).all())
    # the tuned plan: greedy rows take the fp32 argmax up to bf16 rounding of close logits
    tok = ops.lm_head_sample(x, w, temps, step, col_offset)
    ref32 = x.float() @ w.float().t()
    greedy = temps <= 0
    got = ref32.gather(1, (tok.long() - col_offset)[:, None])[:, 0]
    assert bool((got[greedy] >= ref32.max(1).values[greedy] - 0.02).all())
    assert bool((sc.sample_keys[:m] == 0).all())
    assert ops.C.gemm_error(True) == 0


def test_temperature_sampling_never_leaves_the_live_columns(ops):
    """Full-vocabulary rows at T = 1 with 4 live columns: the noise stays finite for every column
    (a noise value of +inf would let a dead column win about once per 2^24 columns)."""
    V, rows = 151936, 4096
    base = torch.full((V,), -30.0, device=DEV)
    cols = torch.tensor([11, 5000, 70000, 151935], device=DEV)
    base[cols] = torch.log(torch.tensor([0.4, 0.3, 0.2, 0.1], device=DEV))
    logits = base.repeat(rows, 1)
    for s in range(3):
        tok = ops.sample(logits, torch.ones(rows, device=DEV), step=torch.tensor([9, s], dtype=torch.int64, device=DEV))
        assert bool((tok.long()[:, None] == cols[None]).any(1).all())


def test_sample_top_p_on_gpu(ops):
    """Nucleus sampling in one kernel: only the nucleus is drawn, in its renormalised proportions."""
    V, rows = 151936, 4096
    base = torch.full((V,), -30.0, device=DEV)
    probs = torch.tensor([0.4, 0.3, 0.2, 0.1], device=DEV)
    base[[11, 5000, 70000, 151935]] = torch.log(probs)
    logits = base.repeat(rows, 1)
    temps = torch.ones(rows, device=DEV)
    counts = {0.6: torch.zeros(4), 0.95: torch.zeros(4), 1.0: torch.zeros(4)}
    cols = torch.tensor([11, 5000, 70000, 151935], device=DEV)
    for p in counts:
        for s in range(3):
            tok = ops.sample(logits, temps, torch.full((rows,), p, device=DEV),
                             step=torch.tensor([5, s], dtype=torch.int64, device=DEV), use_top_p=True)
            hit = (tok.long()[:, None] == cols[None]).float()
            assert bool((hit.sum(1) == 1).all()), "a token outside the four live columns was drawn"
            counts[p] += hit.sum(0).cpu()
    f = {p: c / c.sum() for p, c in counts.items()}
    assert torch.allclose(f[0.6], torch.tensor([4 / 7, 3 / 7, 0, 0]), atol=0.02), f[0.6]
    assert torch.allclose(f[0.95], torch.tensor([0.4, 0.3, 0.2, 0.1]), atol=0.02), f[0.95]
    assert torch.allclose(f[1.0], torch.tensor([0.4, 0.3, 0.2, 0.1]), atol=0.02), f[1.0]
    # greedy rows in the same launch take the argmax; a row at T -> 0+ with p < 1 too
    t2 = torch.tensor([0.0, 1e-4, 1.0], device=DEV)
    tok = ops.sample(logits[:3], t2, torch.tensor([0.5, 0.5, 1.0], device=DEV),
                     step=torch.tensor([1, 2], dtype=torch.int64, device=DEV), use_top_p=True)
    assert tok[0].item() == 11 and tok[1].item() == 11
    assert ops.C.sample_error(True) == 0


@pytest.mark.parametrize("m,n,k", [
    (1, 1024, 1024), (5, 6144, 4096), (64, 4096, 4096), (130, 24576, 1024), (256, 512, 3072),
    (300, 1024, 1024), (1000, 3072, 1024), (4096, 4096, 4096), (77, 151936, 1024), (2, 768, 4096),
])
def test_gemm_tcgen05(ops, m, n, k):
    g = torch.Generator(device=DEV).manual_seed(m * 7 + n)
    x = (torch.randn(m, k, device=DEV, generator=g) * 0.5).bfloat16()
    w = (torch.randn(n, k, device=DEV, generator=g) * 0.02).bfloat16()
    out = ops.linear(x, w)
    ref = x.float() @ w.float().t()
    _close(out, ref, 0.01 * math.sqrt(k / 1024) * 0.5, 0.02)
    assert ops.C.gemm_error(True) == 0


@pytest.mark.parametrize("m,n,k,act", [
    (1, 6144, 4096, 0), (7, 4096, 512, 0), (16, 4096, 12288, 0), (33, 1536, 2048, 0), (64, 24576, 4096, 1),
    (100, 4096, 4096, 0), (200, 2304, 1024, 0), (256, 6144, 4096, 0), (5, 3072, 1024, 1), (129, 768, 4096, 1),
])
def test_gemm_skinny_configs(ops, m, n, k, act):
    """The skinny kernel (weights on the MMA's M side, 128- or 64-row MMAs, cluster split-K) over its
    top configurations."""
    from nanovllm_self_b200.ops.torch_ref import interleave_gate_up
    g = torch.Generator(device=DEV).manual_seed(m * 13 + n)
    x = (torch.randn(m, k, device=DEV, generator=g) * 0.5).bfloat16()
    w = (torch.randn(n, k, device=DEV, generator=g) * 0.02).bfloat16()
    ref = x.float() @ w.float().t()
    if act:
        gate, up = ref[:, : n // 2], ref[:, n // 2:]
        ref = torch.nn.functional.silu(gate) * up
        w = interleave_gate_up(w[: n // 2], w[n // 2:]).contiguous()
    rows = []  # weight rows per CTA of every configuration run (64: the 64-row MMA shape)
    for rank in range(12):
        out = torch.full((m, n // 2 if act else n), float("nan"), device=DEV, dtype=torch.bfloat16)
        cfg = ops.C.linear_skinny(x, w, out, rank, act)
        if not cfg:
            break
        rows.append(cfg[1])
        _close(out, ref, 0.01 * math.sqrt(k / 1024) * 0.5, 0.02)
    assert rows
    if n // 64 <= 148:  # the 64-row single-split shape fits one wave: it is among the plans
        assert 64 in rows, rows
    assert ops.C.gemm_error(True) == 0


@pytest.mark.parametrize("m,n,k,act", [
    (256, 6144, 4096, 0), (129, 4096, 4096, 0), (200, 24576, 4096, 1), (256, 4096, 12288, 0), (177, 1000, 512, 0),
])
def test_gemm_pair_configs(ops, m, n, k, act):
    """The CTA-pair kernel (M = 256 tokens over two CTAs, cta_group::2) over its top configurations,
    ragged token counts and a ragged last weight tile included."""
    from nanovllm_self_b200.ops.torch_ref import interleave_gate_up
    g = torch.Generator(device=DEV).manual_seed(m * 7 + n)
    x = (torch.randn(m, k, device=DEV, generator=g) * 0.5).bfloat16()
    w = (torch.randn(n, k, device=DEV, generator=g) * 0.02).bfloat16()
    ref = x.float() @ w.float().t()
    if act:
        gate, up = ref[:, : n // 2], ref[:, n // 2:]
        ref = torch.nn.functional.silu(gate) * up
        w = interleave_gate_up(w[: n // 2], w[n // 2:]).contiguous()
    ops.C.gemm_error(True)
    ran = []
    for rank in range(6):
        out = torch.full((m, n // 2 if act else n), float("nan"), device=DEV, dtype=torch.bfloat16)
        cfg = ops.C.linear_pair(x, w, out, rank, act)
        if not cfg:
            break
        torch.cuda.synchronize()
        assert ops.C.gemm_error(True) == 0, cfg
        ran.append(cfg)
        _close(out, ref, 0.01 * math.sqrt(k / 1024) * 0.5, 0.02)
    assert ran


@pytest.mark.parametrize("swap,bn,splits", [(0, 256, 1), (0, 128, 3), (1, 32, 1), (1, 64, 4), (1, 256, 2), (0, 64, 1)])
def test_gemm_forced_configs(ops, swap, bn, splits):
    m, n, k = 200, 1280, 2048
    x = torch.randn(m, k, device=DEV).bfloat16()
    w = (torch.randn(n, k, device=DEV) * 0.05).bfloat16()
    out = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    sc = ops.scratch(x.device)
    ops.C.linear(x, w, out, sc.gemm, sc.gemm_counters, swap, bn, splits)
    assert int(sc.gemm_counters.abs().sum()) == 0  # the fix-up leaves the counters at zero
    _close(out, x.float() @ w.float().t(), 0.05, 0.02)


@pytest.mark.parametrize("m,n,k,bn,mt", [
    (200, 1280, 2048, 256, 2), (200, 1280, 2048, 128, 1), (256, 24576, 1024, 256, 2), (64, 6144, 4096, 256, 1),
    (300, 4096, 12288, 128, 2), (17, 1024, 512, 64, 1),
])
def test_gemm_streamk(ops, m, n, k, bn, mt):
    # stream-K: every CTA takes an equal share of the (tile, k-block) iterations; tiles split
    # across CTAs are summed by their last contributor.  Two launches: the counters must be
    # back at zero after each.
    g = torch.Generator(device=DEV).manual_seed(m + n + k)
    x = torch.randn(m, k, device=DEV, generator=g).bfloat16()
    w = (torch.randn(n, k, device=DEV, generator=g) * 0.05).bfloat16()
    out = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    sc = ops.scratch(x.device)
    ref = x.float() @ w.float().t()
    for _ in range(2):
        out.fill_(0)
        ops.C.linear(x, w, out, sc.gemm, sc.gemm_counters, 0, bn, -mt)
        assert int(sc.gemm_counters.abs().sum()) == 0
        _close(out, ref, 0.05 * math.sqrt(k / 2048), 0.02)
    assert ops.C.gemm_error(True) == 0



@pytest.mark.parametrize("m,n,k", [
    (1, 1280, 1024), (7, 6144, 4096), (64, 4096, 4096), (128, 1000, 2048), (129, 24576, 1024), (200, 4096, 12288),
    (256, 6144, 4096),
])
def test_gemm_decode_kernel(ops, m, n, k):
    # all tokens in one CTA tile, runtime tile width, K split over a cluster: the four
    # cheapest configurations of the cost model, each checked against fp32
    g = torch.Generator(device=DEV).manual_seed(m * 3 + n + k)
    x = torch.randn(m, k, device=DEV, generator=g).bfloat16()
    w = (torch.randn(n, k, device=DEV, generator=g) * 0.05).bfloat16()
    ref = x.float() @ w.float().t()
    seen = 0
    for rank in range(4):
        out = torch.zeros(m, n, device=DEV, dtype=torch.bfloat16)
        cfg = ops.C.linear_dec(x, w, out, rank)
        if not cfg:
            break
        seen += 1
        _close(out, ref, 0.05 * math.sqrt(k / 2048), 0.02)
    assert seen > 0
    assert ops.C.gemm_error(True) == 0


@pytest.mark.parametrize("m,inter,k", [(1, 512, 1024), (64, 1536, 2048), (200, 6144, 4096), (256, 12288, 1024),
                                       (777, 1024, 512)])
def test_gemm_silu_epilogue(ops, m, inter, k):
    # gate/up rows interleaved in groups of 16; every GEMM variant's fused epilogue must
    # give silu(gate) * up
    g = torch.Generator(device=DEV).manual_seed(m + inter)
    x = torch.randn(m, k, device=DEV, generator=g).bfloat16()
    wg = (torch.randn(inter, k, device=DEV, generator=g) * 0.05).bfloat16()
    wu = (torch.randn(inter, k, device=DEV, generator=g) * 0.05).bfloat16()
    w = R.interleave_gate_up(wg, wu).contiguous()
    ref = torch.nn.functional.silu(x.float() @ wg.float().t()) * (x.float() @ wu.float().t())
    sc = ops.scratch(x.device)
    tol = 0.05 * math.sqrt(k / 2048)
    outs = [ops.linear_silu(x, w)]
    for bn, sp in [(256, 1), (128, 3), (128, -1), (256, -2)]:
        o = torch.zeros(m, inter, device=DEV, dtype=torch.bfloat16)
        ops.C.linear(x, w, o, sc.gemm, sc.gemm_counters, 0, bn, sp, 1)
        outs.append(o)
    if m <= 256:
        for rank in range(3):
            o = torch.zeros(m, inter, device=DEV, dtype=torch.bfloat16)
            cfg = ops.C.linear_dec(x, w, o, rank, 1)
            if cfg and cfg[0]:
                outs.append(o)
    for o in outs:
        _close(o, ref, tol, 0.03)
    assert int(sc.gemm_counters.abs().sum()) == 0
    assert ops.C.gemm_error(True) == 0
