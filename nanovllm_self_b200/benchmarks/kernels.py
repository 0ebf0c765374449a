"""Single-kernel cases of the hot ops, timed with CUDA events or run once for a profiler.

``python -m nanovllm_self_b200.benchmarks.kernels <case> [--mode time|profile] [--iters N]``

``--mode time`` (default) runs 3 warm-up launches, then ``--iters`` launches, each after a
read of a 256 MiB buffer (> the 126 MB L2; a read leaves no dirty lines whose write-back
the timed launch would pay for) so that every timed launch reads from HBM, and
prints one JSON line: the median device time, the algorithmic bytes or FLOPs of one launch
and their fraction of the peaks in ``MEASURED_PEAKS.json`` (repository root) when present.
``--mode profile`` runs one untimed launch (which also autotunes the GEMM cases), then
three launches between ``cudaProfilerStart``/``cudaProfilerStop`` and exits: the small
workload a profiler capture of one launch needs (``ncu --profile-from-start off -c 1``).

Shapes are Qwen3-8B's (32 query heads, 8 KV heads, head dim 128, hidden 4096,
intermediate 12288, vocab 151936); every case holds well under 2 GB on the device.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import torch

from ..ops.cuda_ops import CudaOps

NQ, NKV, D, HID, INTER, VOCAB = 32, 8, 128, 4096, 12288, 151936
CASES = ("attn_decode", "attn_decode_fp8", "attn_prefill", "attn_prefill_mma", "attn_prefill_fp8",
         "attn_prefill_flash_attn", "gemm_prefill", "gemm_decode", "gemm_decode256", "gemm_gate_up_silu256", "qkv_post",
         "qkv_post_fp8", "add_rmsnorm", "silu_mul", "sample", "qkv_post256", "lm_head_sample256", "lm_head_logits_sample256",
         "lm_head_sample256_t", "lm_head_logits_sample256_t", "lm_head_logits256")
# Qwen3-8B decode GEMM shapes (n, k) for gemm_sweep: qkv, o_proj, gate_up, down_proj, lm_head
DECODE_SHAPES = {"qkv": ((NQ + 2 * NKV) * D, HID), "o_proj": (HID, NQ * D), "gate_up": (2 * INTER, HID),
                 "down_proj": (HID, INTER), "lm_head": (VOCAB, HID)}


class _Ctx:
    pass


def _paged(B, ctx_len, qlen, fp8, dev, bs=256):
    nbps = (ctx_len + bs - 1) // bs
    nb = B * nbps + 1
    kc = torch.randn(nb, NKV, bs, D, device=dev).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    ks = vs = None
    if fp8:
        kc, vc = kc.to(torch.float8_e4m3fn), vc.to(torch.float8_e4m3fn)
        ks = torch.full((nb, NKV), 1.0, device=dev)
        vs = torch.full((nb, NKV), 1.0, device=dev)
    c = _Ctx()
    c.block_tables = torch.arange(B * nbps, device=dev, dtype=torch.int32).view(B, nbps)
    c.cu_seqlens_q = torch.arange(0, B * qlen + 1, qlen, device=dev, dtype=torch.int32)
    c.context_lens = torch.full((B,), ctx_len, device=dev, dtype=torch.int32)
    c.max_seqlen_q, c.max_seqlen_k = qlen, ctx_len
    c.num_decode_seqs = B if qlen == 1 else 0
    c.num_seqs = B
    q = torch.randn(B * qlen, NQ * D, device=dev).to(torch.bfloat16)
    return q, kc, vc, ks, vs, c


def build_case(name: str, ops: CudaOps, dev="cuda"):
    """Returns (launch, bytes, flops) for one case; ``launch()`` runs the op once."""
    torch.manual_seed(0)
    if name.startswith("attn_decode"):
        fp8 = name.endswith("fp8")
        B, L = 128, 2048
        q, kc, vc, ks, vs, c = _paged(B, L, 1, fp8, dev)
        kv_bytes = 2 * B * NKV * L * D * kc.element_size()
        return (lambda: ops.attention(q, kc, vc, c, D ** -0.5, ks, vs)), kv_bytes + 2 * q.numel() * 2, \
            4 * B * NQ * L * D
    if name == "attn_prefill_flash_attn":
        # the reference's prefill kernel (flash_attn_varlen_func, causal, contiguous K/V), same shape
        from flash_attn import flash_attn_varlen_func
        B, L = 8, 2048
        q = torch.randn(B * L, NQ, D, device=dev).to(torch.bfloat16)
        k = torch.randn(B * L, NKV, D, device=dev).to(torch.bfloat16)
        v = torch.randn_like(k)
        cu = torch.arange(0, B * L + 1, L, device=dev, dtype=torch.int32)
        return (lambda: flash_attn_varlen_func(q, k, v, cu, cu, L, L, causal=True, softmax_scale=D ** -0.5)), None, \
            2 * B * NQ * L * L * D
    if name.startswith("attn_prefill"):
        fp8 = name.endswith("fp8")
        B, L = 8, 2048
        q, kc, vc, ks, vs, c = _paged(B, L, L, fp8, dev)
        ops.prefill_tc = name != "attn_prefill_mma"
        return (lambda: ops.attention(q, kc, vc, c, D ** -0.5, ks, vs)), None, 2 * B * NQ * L * L * D
    if name == "gemm_gate_up_silu256":
        from ..ops.torch_ref import interleave_gate_up
        m = 256
        x = torch.randn(m, HID, device=dev).to(torch.bfloat16)
        w = interleave_gate_up(*(torch.randn(2, INTER, HID, device=dev) * 0.02).to(torch.bfloat16)).contiguous()
        return (lambda: ops.linear_silu(x, w)), 2 * (m * HID + 2 * INTER * HID + m * INTER), 2 * m * 2 * INTER * HID
    if name.startswith("gemm"):
        m, n, k = {"gemm_prefill": (4096, 2 * INTER, HID), "gemm_decode": (64, (NQ + 2 * NKV) * D, HID),
                   "gemm_decode256": (256, 2 * INTER, HID)}[name]
        x = torch.randn(m, k, device=dev).to(torch.bfloat16)
        w = (torch.randn(n, k, device=dev) * 0.02).to(torch.bfloat16)
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        return (lambda: ops.linear(x, w, out)), 2 * (m * k + n * k + m * n), 2 * m * n * k
    if name.startswith("qkv_post"):
        from ..ops.torch_ref import rope_cos_sin
        fp8 = name.endswith("fp8")
        T = 256 if name == "qkv_post256" else 16384  # a 256-sequence decode step, or a prefill chunk
        qkv = torch.randn(T, (NQ + 2 * NKV) * D, device=dev).to(torch.bfloat16)
        nb = T // 256 + 1
        kdt = torch.float8_e4m3fn if fp8 else torch.bfloat16
        kc = torch.zeros(nb, NKV, 256, D, device=dev, dtype=kdt)
        vc = torch.zeros_like(kc)
        ks = torch.ones(nb, NKV, device=dev) if fp8 else None
        vs = torch.ones(nb, NKV, device=dev) if fp8 else None
        pos = torch.arange(T, device=dev, dtype=torch.int32) % 2048
        slots = torch.arange(T, device=dev, dtype=torch.int32)
        cs = rope_cos_sin(D, 4096, 1e6, device=dev)
        w = torch.ones(D, device=dev, dtype=torch.bfloat16)
        nbytes = qkv.numel() * 2 + T * NQ * D * 2 + 2 * T * NKV * D * kc.element_size()
        return (lambda: ops.qkv_post(qkv, w, w, 1e-6, pos, cs, kc, vc, slots, ks, vs, NQ, NKV, D)), nbytes, None
    if name == "add_rmsnorm":
        x = torch.randn(16384, HID, device=dev).to(torch.bfloat16)
        r = torch.randn_like(x)
        w = torch.ones(HID, device=dev, dtype=torch.bfloat16)
        return (lambda: ops.add_rmsnorm(x, r, w, 1e-6)), 4 * x.numel() * 2, None
    if name == "silu_mul":
        x = torch.randn(8192, 2 * INTER, device=dev).to(torch.bfloat16)
        return (lambda: ops.silu_mul(x)), x.numel() * 2 * 3 // 2, None
    if name == "sample":
        logits = torch.randn(256, VOCAB, device=dev).to(torch.bfloat16)
        t = torch.zeros(256, device=dev)
        st = torch.tensor([0, 1], dtype=torch.int64, device=dev)
        return (lambda: ops.sample(logits, t, step=st)), logits.numel() * 2, None
    if name.startswith("lm_head"):
        # Qwen3-8B lm_head at a 256-token decode step, greedy (or, "_t", every row at temperature
        # 0.8): the sampler in the GEMM epilogue ("lm_head_sample256"), the GEMM writing bf16 logits
        # followed by the sampler kernel ("lm_head_logits_sample256"), or the GEMM alone
        m = 256
        x = torch.randn(m, HID, device=dev).to(torch.bfloat16)
        w = (torch.randn(VOCAB, HID, device=dev) * 0.02).to(torch.bfloat16)
        t = torch.full((m,), 0.8 if name.endswith("_t") else 0.0, device=dev)
        st = torch.tensor([0, 1], dtype=torch.int64, device=dev)
        wbytes = 2 * (m * HID + VOCAB * HID)
        if name.startswith("lm_head_sample256"):
            return (lambda: ops.lm_head_sample(x, w, t, st)), wbytes, 2 * m * VOCAB * HID
        out = torch.empty(m, VOCAB, device=dev, dtype=torch.bfloat16)
        if name == "lm_head_logits256":
            return (lambda: ops.linear(x, w, out)), wbytes + 2 * m * VOCAB, 2 * m * VOCAB * HID
        return (lambda: ops.sample(ops.linear(x, w, out), t, step=st)), wbytes, 2 * m * VOCAB * HID
    raise ValueError(f"unknown case {name!r}; one of {', '.join(CASES)}")


def _peaks():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def time_case(name: str, iters: int = 20) -> dict:
    ops = CudaOps()
    launch, nbytes, flops = build_case(name, ops)
    flush = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush.sum()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        launch()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    us = statistics.median(times)
    hbm, tfl, src = _peaks()
    out = {"case": name, "us": round(us, 2), "iters": iters, "l2": "256 MiB read before each launch",
           "peaks": src}
    if name.startswith("gemm"):
        # splits < 0: stream-K with -splits token sub-tiles; splits >= 100: decode kernel, splits - 100 K slices
        out["plan"] = dict(zip(("swap", "bn", "tiles_p", "tiles_q", "splits", "grid"), ops.last_plan))
    if nbytes:
        out["gb_s"] = round(nbytes / us / 1e3, 1)
        out["frac_hbm"] = round(nbytes / us / 1e3 / hbm, 3)
    if flops:
        out["tflops"] = round(flops / us / 1e6, 1)
        out["frac_bf16"] = round(flops / us / 1e6 / tfl, 3)
    return out


def gemm_sweep(ms=(1, 16, 64, 128, 256), iters: int = 20) -> None:
    """Our tcgen05 GEMM (autotuned) against cuBLAS (torch.matmul) on the Qwen3-8B decode shapes.

    One JSON line per (shape, m): median CUDA-event time of each over `iters` launches, every
    launch after a 256 MiB read (cold L2, as when a layer's weights are used in a forward).
    """
    ops = CudaOps()
    flush = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    hbm, tfl, src = _peaks()

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(iters):
            flush.sum()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        return statistics.median(ts)

    for name, (n, k) in DECODE_SHAPES.items():
        w = (torch.randn(n, k, device="cuda") * 0.02).to(torch.bfloat16)
        for m in ms:
            x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
            out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
            ours = timed(lambda: ops.linear(x, w, out))
            plan = dict(zip(("swap", "bn", "tiles_p", "tiles_q", "splits", "grid"), ops.last_plan))
            cublas = timed(lambda: torch.matmul(x, w.t(), out=out))
            nbytes = 2 * (m * k + n * k + m * n)
            roof = max(nbytes / (hbm * 1e3), 2 * m * n * k / (tfl * 1e6))
            print(json.dumps({"shape": name, "m": m, "n": n, "k": k, "ours_us": round(ours, 2),
                              "cublas_us": round(cublas, 2), "ours_vs_cublas": round(cublas / ours, 3),
                              "roofline_us": round(roof, 2), "frac_roofline": round(roof / ours, 3), "plan": plan,
                              "l2": "256 MiB read before each launch", "peaks": src}), flush=True)
        del w


def gemm_chain(ms=(1, 16, 64, 128, 256), calls: int = 24) -> None:
    """Decode GEMMs as the engine runs them: `calls` back-to-back launches captured in one CUDA
    graph (programmatic dependent launch lets each GEMM's weight stream start while the previous
    kernel finishes), weights rotating over enough copies to exceed the L2.  Per-call time =
    graph replay time / calls; ours (autotuned) against cuBLAS (torch.matmul) in the same form."""
    ops = CudaOps()
    hbm, tfl, src = _peaks()
    for name, (n, k) in DECODE_SHAPES.items():
        if name == "lm_head":
            continue
        wbytes = n * k * 2
        copies = max(2, min(calls, (384 << 20) // wbytes + 1))
        ws = [(torch.randn(n, k, device="cuda") * 0.02).to(torch.bfloat16) for _ in range(copies)]
        for m in ms:
            x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
            out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
            res = {}
            for impl in ("ours", "cublas"):
                def body():
                    for i in range(calls):
                        if impl == "ours":
                            ops.linear(x, ws[i % copies], out)
                        else:
                            torch.matmul(x, ws[i % copies].t(), out=out)
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(s):
                    body()  # tunes outside the capture
                torch.cuda.current_stream().wait_stream(s)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    body()
                for _ in range(3):
                    g.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(5):
                    g.replay()
                e1.record()
                torch.cuda.synchronize()
                res[impl] = e0.elapsed_time(e1) * 1e3 / (5 * calls)
                del g
            roof = max(2 * (m * k + n * k + m * n) / (hbm * 1e3), 2 * m * n * k / (tfl * 1e6))
            print(json.dumps({"shape": name, "m": m, "n": n, "k": k, "ours_us": round(res["ours"], 2),
                              "cublas_us": round(res["cublas"], 2), "ours_vs_cublas": round(res["cublas"] / res["ours"], 3),
                              "roofline_us": round(roof, 2), "frac_roofline": round(roof / res["ours"], 3),
                              "plan": dict(zip(("swap", "bn", "tiles_p", "tiles_q", "splits", "grid"), ops.last_plan)),
                              "timing": f"CUDA graph of {calls} calls, weights rotating over {copies} copies",
                              "peaks": src}), flush=True)
        del ws


def gemm_one(m: int, n: int, k: int, impl: str, mode: str, iters: int = 20) -> None:
    """One GEMM shape with one implementation: ``tuned`` (the autotuner's pick), ``cublas``
    (torch.matmul), ``skinny:R`` / ``dec:R`` / ``pair:R`` (the R-th configuration of that kernel's model)."""
    ops = CudaOps()
    x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda") * 0.02).to(torch.bfloat16)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    kind, _, rank = impl.partition(":")
    info = {}
    if kind == "tuned":
        def fn():
            ops.linear(x, w, out)
    elif kind == "cublas":
        def fn():
            torch.matmul(x, w.t(), out=out)
    elif kind == "skinny":
        def fn():
            info["cfg"] = ops.C.linear_skinny(x, w, out, int(rank or 0), 0)
    elif kind == "skinnyb":  # weights in the blocked [n/128, k/64, 128, 64] layout
        wb = w.view(n // 128, 128, k // 64, 64).permute(0, 2, 1, 3).contiguous()

        def fn():
            info["cfg"] = ops.C.linear_skinny(x, wb, out, int(rank or 0), 0, 1)
    elif kind == "dec":
        def fn():
            info["cfg"] = ops.C.linear_dec(x, w, out, int(rank or 0), 0)
    elif kind == "pair":  # CTA-pair kernel (128 < m <= 256)
        def fn():
            info["cfg"] = ops.C.linear_pair(x, w, out, int(rank or 0), 0)
    else:
        raise ValueError(impl)
    fn()
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    err = ((out.float() - ref).abs().max() / ref.abs().max()).item()
    if mode == "profile":
        torch.cuda.profiler.start()
        fn()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"gemm": [m, n, k], "impl": impl, "profiled_launches": 1, "rel_err": err, **info}))
        return
    flush = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    ts = []
    for _ in range(iters):
        flush.sum()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3)
    print(json.dumps({"gemm": [m, n, k], "impl": impl, "us": round(statistics.median(ts), 2), "rel_err": err,
                      "plan": ops.last_plan if kind == "tuned" else info.get("cfg")}))


def skinny_trace(m: int, n: int, k: int, rank: int) -> None:
    """In-kernel %globaltimer stamps of one cold launch of the rank-th skinny configuration: per CTA,
    when each k-block's loads were issued and when the MMA thread saw them land."""
    ops = CudaOps()
    x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda") * 0.02).to(torch.bfloat16)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    cfg = ops.C.linear_skinny(x, w, out, rank, 0)  # warm-up
    tr = torch.zeros(4096 * 328, dtype=torch.int64, device="cuda")
    flush = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    flush.sum()
    ops.C.linear_skinny(x, w, out, rank, 0, 0, tr)
    torch.cuda.synchronize()
    t = tr.view(4096, 328).cpu()
    live = t[:, 0] > 0
    t = t[live]
    t0 = t[:, 0].min()
    lat, gaps, land, waited, busy, mma, com, tail = [], [], [], [], [], [], [], []
    for row in t:
        issue = row[8:72]
        full = row[72:136]
        start = row[136:200]
        after_mma = row[200:264]
        after_com = row[264:328]
        for i in range(64):
            if full[i] > 0 and after_mma[i] > 0 and after_com[i] > 0:
                mma.append(int(after_mma[i] - full[i]))     # fence + MMA issue (+ one stamp)
                com.append(int(after_com[i] - after_mma[i]))  # commit issue (+ one stamp)
            if i < 63 and after_com[i] > 0 and start[i + 1] > 0:
                tail.append(int(start[i + 1] - after_com[i]))  # loop overhead to the next wait
        for i in range(64):
            if issue[i] > 0 and full[i] > 0:
                lat.append(int(full[i] - issue[i]))
            if i > 0 and full[i] > 0 and full[i - 1] > 0:
                land.append(int(full[i] - full[i - 1]))
                busy.append(int(start[i] - full[i - 1]))  # MMA thread's own work for k-block i - 1
            if full[i] > 0 and start[i] > 0:
                waited.append(int(full[i] - start[i]))  # how long it waited for k-block i
    q = lambda v, p: float(torch.tensor(v, dtype=torch.float64).quantile(p)) / 1e3 if v else None
    print(json.dumps({"gemm": [m, n, k], "cfg": cfg, "ctas": int(live.sum()),
                      "first_full_us": q([int(r[2] - t0) for r in t], 0.5),
                      "mma_done_us_p50": q([int(r[3] - t0) for r in t if r[3] > 0], 0.5),
                      "end_us_max": q([int(r[6] - t0) for r in t], 1.0),
                      "issue_to_land_us": {"p10": q(lat, 0.1), "p50": q(lat, 0.5), "p90": q(lat, 0.9)},
                      "land_to_land_us": {"p10": q(land, 0.1), "p50": q(land, 0.5), "p90": q(land, 0.9)},
                      "mma_thread_work_us": {"p10": q(busy, 0.1), "p50": q(busy, 0.5), "p90": q(busy, 0.9)},
                      "mma_thread_wait_us": {"p10": q(waited, 0.1), "p50": q(waited, 0.5), "p90": q(waited, 0.9)},
                      "mma_issue_us_p50": q(mma, 0.5), "commit_issue_us_p50": q(com, 0.5), "loop_tail_us_p50": q(tail, 0.5)}))


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("case", choices=CASES + ("all", "gemm_sweep", "gemm_one", "gemm_chain", "skinny_trace"))
    p.add_argument("--rank", type=int, default=0)
    p.add_argument("--m", type=int, default=1)
    p.add_argument("--n", type=int, default=6144)
    p.add_argument("--k", type=int, default=4096)
    p.add_argument("--impl", default="tuned", help="comma-separated: tuned, cublas, skinny:R, skinnyb:R, dec:R, pair:R")
    p.add_argument("--ms", default=None, help="comma-separated m values (gemm_one), instead of --m")
    p.add_argument("--mode", choices=("time", "profile"), default="time")
    p.add_argument("--iters", type=int, default=20)
    a = p.parse_args(argv)
    if a.case == "gemm_sweep":
        gemm_sweep(iters=a.iters)
        return
    if a.case == "gemm_chain":
        gemm_chain()
        return
    if a.case == "skinny_trace":
        skinny_trace(a.m, a.n, a.k, a.rank)
        return
    if a.case == "gemm_one":
        for impl in a.impl.split(","):
            for m in (a.ms.split(",") if a.ms else [a.m]):
                gemm_one(int(m), a.n, a.k, impl, a.mode, a.iters)
        return
    names = CASES if a.case == "all" else (a.case,)
    for n in names:
        if a.mode == "profile":
            launch = build_case(n, CudaOps())[0]
            launch()
            torch.cuda.synchronize()
            torch.cuda.profiler.start()
            for _ in range(3):
                launch()
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
            print(json.dumps({"case": n, "profiled_launches": 3}), flush=True)
        else:
            print(json.dumps(time_case(n, a.iters)), flush=True)


if __name__ == "__main__":
    main()
