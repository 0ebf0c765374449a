// Persistent bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Computes C = X * W^T for every linear layer of the model (the reference runs these
// as nn.Linear / cuBLAS: q/k/v/o projections nanovllm/models/qwen3.py:96-120,
// gate/up/down :131-134, lm_head :508).  Both operands are K-major ("TN"), which is
// the native operand layout of tcgen05.mma, so no transposes are needed.
//
// The kernel computes D[i, j] = sum_k P[i, k] * Q[j, k] on tiles of 128 (P rows, one
// TMEM lane each) x BN (Q rows, TMEM columns):
//   * normal mode (prefill): P = X (tokens), Q = W (features), C[i, j] = D[i, j];
//   * swap mode (decode, few tokens): P = W, Q = X, C[j, i] = D[i, j], so a batch of
//     1..256 tokens still fills the 128-row MMA with weight rows.
//
// Warp roles (192 threads, one CTA per SM, persistent over output tiles x K splits):
//   warp 0: TMA producer into a STAGES-deep shared-memory ring (128B swizzle);
//   warp 1: TMEM allocator + single-thread MMA issuer (tcgen05.mma kind::f16, M=128);
//   warps 2-5: epilogue; tcgen05.ld of the fp32 accumulator, convert, store.
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue of tile
// t overlaps the main loop of tile t+1.  Problems with too few output tiles to fill the
// GPU (decode projections) use gemm_cluster_kernel instead: split-K across the CTAs of
// a thread-block cluster, reduced through distributed shared memory.
//
// Every mbarrier wait is bounded by a wall-clock budget; on expiry the kernel records
// an error code in a device word (read by gemm_error_code()), stops issuing work,
// drains its own copies and MMAs with bounded waits, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "common.cuh"
#include "gemm.h"

namespace nvb {

__device__ int g_gemm_error = 0;

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int NUM_THREADS = 192;
constexpr uint64_t WAIT_BUDGET_NS = 2000000000ull;  // 2 s
constexpr int PF_DIST = 12;                          // k-blocks of L2 prefetch lookahead

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait.  Returns false (after recording `code`) if the budget expires or another
// role of this CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int code) {
  if (mbar_try(bar, parity)) return true;
  SpinBudget sb;
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return false;
    if (sb.expired(WAIT_BUDGET_NS)) {
      atomicCAS(&g_gemm_error, 0, code);
      *abort_flag = 1;
      return false;
    }
  }
}

// Bounded wait for a long phase (the epilogue warps waiting for the whole mainloop): polls
// with a back-off so the spinning warps leave the issue slots to the producer and MMA threads
// that share their SM sub-partitions.
__device__ __forceinline__ bool mbar_wait_sleep(uint32_t bar, uint32_t parity, volatile int* abort_flag, int code) {
  if (mbar_try(bar, parity)) return true;
  SpinBudget sb;
  while (true) {
    __nanosleep(128);
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return false;
    if (sb.expired(WAIT_BUDGET_NS)) {
      atomicCAS(&g_gemm_error, 0, code);
      *abort_flag = 1;
      return false;
    }
  }
}

// Drain wait used on the error path: short budget, never sets flags.
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
  SpinBudget sb;
  while (!mbar_try(bar, parity)) {
    if (sb.expired(WAIT_BUDGET_NS)) return;
  }
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// Pull a tile of the streamed (weight) operand into L2 ahead of its TMA load, so the
// ring's loads see L2 latency instead of HBM latency.
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// tcgen05 fences order tcgen05 operations against thread synchronisation (an mbarrier that other
// threads arrive on after their own tcgen05 work, or __syncthreads).  The mainloops issue MMAs right
// after waiting on a TMA-filled stage barrier without one: that wait already orders the staged data.
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
  d |= (uint64_t)1 << 46;             // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

template <int BN>
__device__ __forceinline__ constexpr uint32_t idesc_bf16() {
  return (1u << 4)                          // D format f32
         | (1u << 7)                        // A bf16
         | (1u << 10)                       // B bf16
         | ((uint32_t)(BN >> 3) << 17)      // N
         | ((uint32_t)(BM >> 4) << 24);     // M
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct Params {
  int p_rows, q_rows, k;
  int tiles_p, tiles_q, splits, kb_per_split, num_kb;
  int swap;
  int prefetch_w;            // 1: pull weight k-blocks into L2 ahead (decode-sized problems)
  int group;                 // tile rasterisation group along P
  __nv_bfloat16* c;
  int64_t ldc;
  float* ws;                 // split-K partials [splits][p_rows][q_rows_pad]
  int64_t ws_ld;
  int* counters;             // split-K arrival counters, 4 per tile (zero between launches)
  int streamk;               // 1: stream-K split of tiles x k-blocks over the grid
  int64_t sk_iters;          // stream-K: tiles * num_kb
  int act;                   // 1: SiLU-and-mul epilogue (see act_silu_store)
  // Sampling epilogue (lm_head; keys != nullptr): C is not stored.  Each output value is rounded
  // to bf16 (the logit the sampler would read), noised for rows at temperature > 0 (Gumbel-max,
  // the sampler kernels' noise), and folded into keys[token] with an atomic max of
  // (orderable score << 32 | ~global column): the maximum is the sampled token, the lowest column
  // winning ties.  keys is all zero before the launch; sample_keys decodes and re-zeroes it.
  unsigned long long* keys;
  const float* temps;        // [m] temperature per token row (<= 0: greedy)
  const int64_t* seed_step;  // (seed, step) of the sampler noise
  int64_t col_offset;        // global column of output feature 0 (vocab shard start)
};

// Order-preserving map of a float onto uint32; NaN and -inf -> 0, which never wins (the sampler
// kernels skip them too: a row with no finite score gets token 0).
__device__ __forceinline__ uint32_t orderable(float v) {
  const uint32_t u = __float_as_uint(v);
  return (v != v || v == -INFINITY) ? 0u : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
}

// Sampling epilogue of 32 accumulator columns [qc, qc + 32) of accumulator row pi (see Params).
// swap: rows are vocabulary features (a warp's lanes hold 32 consecutive ones) and columns are
// tokens; per column the warp takes the maximum of the order-preserving score words with one
// redux.sync and the first lane holding it with a ballot (the 32 columns are independent, so the
// reductions overlap), and lane j issues the atomic for token qc + j.  Otherwise row pi is a token
// and the thread reduces its 32 features itself.  Called by all 32 lanes of a warp together.
__device__ __forceinline__ void sample_chunk(const Params& p, int pi, int qc, const float* f) {
  const uint64_t seed = (uint64_t)p.seed_step[0], step = (uint64_t)p.seed_step[1];
  if (!p.swap) {
    if (pi >= p.p_rows) return;
    const float t = p.temps[pi];
    const bool greedy = !(t > 0.f);
    const float inv_t = greedy ? 1.f : 1.f / t;
    uint32_t best = 0u;
    int bc = -1;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int c = qc + j;
      if (c >= p.q_rows) break;
      float v = bf16_round(f[j]);
      if (!greedy) v = noised(v, inv_t, seed, step, pi, p.col_offset + c);
      const uint32_t u = orderable(v);
      if (u > best) {
        best = u;
        bc = c;
      }
    }
    if (bc >= 0)
      atomicMax(p.keys + pi, ((unsigned long long)best << 32) | (0xFFFFFFFFu - (uint32_t)(p.col_offset + bc)));
    return;
  }
  const int lane = threadIdx.x & 31;
  const bool row_ok = pi < p.p_rows;
  const int my_tok = qc + lane;
  const float my_t = my_tok < p.q_rows ? p.temps[my_tok] : 0.f;
  const int ncol = min(32, p.q_rows - qc);  // uniform over the warp
  uint32_t my_best = 0u;
  int my_src = -1;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j >= ncol) break;
    const float t = __shfl_sync(FULL_MASK, my_t, j);
    uint32_t u = 0u;
    if (row_ok) {
      float v = bf16_round(f[j]);
      if (t > 0.f) v = noised(v, 1.f / t, seed, step, qc + j, p.col_offset + pi);
      u = orderable(v);
    }
    const uint32_t umax = __reduce_max_sync(FULL_MASK, u);
    const unsigned b = __ballot_sync(FULL_MASK, u == umax);
    if (lane == j) {
      my_best = umax;
      my_src = __ffs(b) - 1;
    }
  }
  if (lane < ncol && my_best != 0u)
    atomicMax(p.keys + my_tok,
              ((unsigned long long)my_best << 32) | (0xFFFFFFFFu - (uint32_t)(p.col_offset + (pi - lane) + my_src)));
}

// Fused SiLU-and-mul epilogue.  The weight rows of a gate/up projection are interleaved
// in groups of 16 (rows 32j..32j+15 = gate features 16j.., rows 32j+16..32j+31 = the
// matching up features), so every 32-column accumulator chunk that starts at a multiple
// of 32 holds 16 gates and their 16 ups: out[16j + i] = silu(g_i) * u_i.
__device__ __forceinline__ float silu_f(float g) { return g / (1.f + expf(-g)); }
__device__ __forceinline__ void act_silu_store(__nv_bfloat16* dst, const float* f) {
  float o[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i] = silu_f(f[i]) * f[16 + i];
  *reinterpret_cast<uint4*>(dst) = f32_to_bf16x8(o);
  *reinterpret_cast<uint4*>(dst + 8) = f32_to_bf16x8(o + 8);
}

__device__ __forceinline__ void unit_coords(const Params& p, int unit, int& tp, int& tq, int& split) {
  const int tiles = p.tiles_p * p.tiles_q;
  split = unit / tiles;
  int t = unit - split * tiles;
  // grouped rasterisation: walk `group` P tiles for each Q tile, so concurrently running
  // CTAs share operand tiles in L2.
  const int per_group = p.group * p.tiles_q;
  const int g = t / per_group;
  const int first_p = g * p.group;
  const int gsize = min(p.group, p.tiles_p - first_p);
  const int r = t - g * per_group;
  tp = first_p + r % gsize;
  tq = r / gsize;
}

// Store 32 accumulator columns [qc, qc + 32) of accumulator row pi as bf16 (or, with the sampling
// epilogue, fold them into the per-token keys).
__device__ __forceinline__ void store_chunk(const Params& p, int pi, int qc, const float* f) {
  if (p.keys) {
    sample_chunk(p, pi, qc, f);
    return;
  }
  if (pi >= p.p_rows) return;
  if (p.act) {  // normal orientation only; q_rows % 32 == 0
    if (qc < p.q_rows) act_silu_store(p.c + (int64_t)pi * p.ldc + qc / 2, f);
    return;
  }
  if (!p.swap) {
    __nv_bfloat16* dst = p.c + (int64_t)pi * p.ldc + qc;
    const int valid = p.q_rows - qc;
    if (valid >= 32) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) *reinterpret_cast<uint4*>(dst + j) = f32_to_bf16x8(f + j);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < valid) dst[j] = __float2bfloat16(f[j]);
    }
  } else {
    // C[j, pi]: the 32 lanes of a warp hold consecutive pi, so each store is coalesced
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (qc + j < p.q_rows) p.c[(int64_t)(qc + j) * p.ldc + pi] = __float2bfloat16(f[j]);
  }
}

// Stream-K work split: CTA c owns iterations [sk_start(c), sk_start(c + 1)) of the
// (tile, k-block) space, so every CTA streams the same number of k-blocks whatever the
// tile count.  A tile whose k-blocks span several CTAs is finished by the last CTA to
// deposit its fp32 partial (arrival counted per epilogue warp): nobody waits on another CTA.
__device__ __forceinline__ int64_t sk_start(const Params& p, int c) {
  return (int64_t)c * p.sk_iters / gridDim.x;
}
// The CTA whose range holds iteration x: the largest c with sk_start(c) <= x.
__device__ __forceinline__ int sk_owner(const Params& p, int64_t x) {
  return (int)(((x + 1) * (int64_t)gridDim.x + p.sk_iters - 1) / p.sk_iters) - 1;
}

// k-blocks [k0, k1) of output tile (tp, tq): one unit of a CTA's work.
struct Seg {
  int tp, tq, k0, k1, tile, slot;
  bool full;  // covers the whole K range (no partial sums)
};

struct SegIter {
  int64_t i, e;
  int u;
  bool first;
  __device__ __forceinline__ void init(const Params& p) {
    if (p.streamk) {
      i = sk_start(p, blockIdx.x);
      e = sk_start(p, blockIdx.x + 1);
    }
    u = blockIdx.x;
    first = true;
  }
  __device__ __forceinline__ bool next(const Params& p, Seg& s) {
    int sp;
    if (p.streamk) {
      if (i >= e) return false;
      const int t = (int)(i / p.num_kb);
      s.k0 = (int)(i - (int64_t)t * p.num_kb);
      s.k1 = (int)min((int64_t)p.num_kb, (int64_t)s.k0 + (e - i));
      s.tile = t;
      unit_coords(p, t, s.tp, s.tq, sp);
      s.full = s.k0 == 0 && s.k1 == p.num_kb;
      s.slot = blockIdx.x * 2 + (first ? 0 : 1);
      i += s.k1 - s.k0;
      first = false;
      return true;
    }
    if (u >= p.tiles_p * p.tiles_q * p.splits) return false;
    unit_coords(p, u, s.tp, s.tq, sp);
    s.k0 = sp * p.kb_per_split;
    s.k1 = min(p.num_kb, s.k0 + p.kb_per_split);
    s.tile = u;
    s.slot = 0;
    s.full = true;
    u += gridDim.x;
    return true;
  }
};

// MT = 128-row P sub-tiles per output tile (2: one CTA covers 256 tokens, so each weight
// k-block it loads feeds two MMAs).  The fp32 accumulators are double-buffered in TMEM
// when both buffers fit in its 512 columns.
template <int BN, int STAGES, int MT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_p, const __grid_constant__ CUtensorMap map_q, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int P_BYTES = BM * BK * 2;
  constexpr int Q_BYTES = BN * BK * 2;
  constexpr int STAGE_BYTES = MT * P_BYTES + Q_BYTES;
  constexpr int ACC_COLS = MT * BN;
  constexpr int ACC_BUFS = 2 * ACC_COLS <= 512 ? 2 : 1;
  constexpr uint32_t TMEM_COLS = ACC_BUFS * ACC_COLS;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  // bars: full[STAGES], empty[STAGES], tfull[2], tempty[2], final
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * STAGES + 5);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 6);
  const uint32_t bar0 = smem_u32(bars);
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
  const uint32_t final_bar = bar0 + 8u * (2 * STAGES + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(tfull(0), 1);
    mbar_init(tfull(1), 1);
    mbar_init(tempty(0), 4);
    mbar_init(tempty(1), 4);
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // inputs and the output may belong to the previous kernel in the stream
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_p)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_q)) : "memory");
      uint32_t it = 0;
      bool ok = true;
      SegIter si;
      si.init(p);
      Seg sg;
      while (ok && si.next(p, sg)) {
        const int nkb = sg.k1 - sg.k0;
        const int rot = p.streamk ? 0 : (sg.tp + sg.tq) % nkb;
        const CUtensorMap* wmap = p.swap ? &map_p : &map_q;
        const int wrow = p.swap ? sg.tp * MT * BM : sg.tq * BN;
        if (p.prefetch_w)
          for (int i = 0; i < min(nkb, PF_DIST); ++i) tma_prefetch_2d(wmap, (sg.k0 + (i + rot) % nkb) * BK, wrow);
        for (int i = 0; i < nkb; ++i, ++it) {
          const int kb = sg.k0 + (i + rot) % nkb;
          const int s = it % STAGES;
          const uint32_t round = it / STAGES;
          if (p.prefetch_w && i + PF_DIST < nkb)
            tma_prefetch_2d(wmap, (sg.k0 + (i + PF_DIST + rot) % nkb) * BK, wrow);
          if (!mbar_wait(empty(s), (round & 1) ^ 1, abort_flag, 1)) {
            ok = false;
            break;
          }
          const uint32_t st = smem_u32(smem + s * STAGE_BYTES);
          mbar_arrive_expect_tx(full(s), STAGE_BYTES);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
            tma_load_2d(st + mt * P_BYTES, &map_p, full(s), kb * BK, (sg.tp * MT + mt) * BM);
          tma_load_2d(st + MT * P_BYTES, &map_q, full(s), kb * BK, sg.tq * BN);
        }
      }
      if (!ok) {
        // Error path: wait (bounded) for copies this thread issued and nobody consumed.
        const uint32_t n = it < (uint32_t)STAGES ? it : (uint32_t)STAGES;
        for (uint32_t j = it - n; j < it; ++j) mbar_drain(full(j % STAGES), (j / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16<BN>();
      uint32_t it = 0, tile_it = 0;
      bool ok = true;
      SegIter si;
      si.init(p);
      Seg sg;
      while (ok && si.next(p, sg)) {
        const int nkb = sg.k1 - sg.k0;
        const int acc = ACC_BUFS == 2 ? (tile_it & 1) : 0;
        const uint32_t use = ACC_BUFS == 2 ? (tile_it >> 1) : tile_it;
        if (!mbar_wait(tempty(acc), (use & 1) ^ 1, abort_flag, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
        for (int i = 0; i < nkb; ++i, ++it) {
          const int s = it % STAGES;
          const uint32_t round = it / STAGES;
          if (!mbar_wait(full(s), round & 1, abort_flag, 3)) {
            ok = false;
            break;
          }
          const uint32_t st = smem_u32(smem + s * STAGE_BYTES);
          const uint64_t qd = sdesc(st + MT * P_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // advance 16 elements (32 bytes) along K inside the swizzle atom: +2 in the
            // 16-byte-unit start address field
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
              tc_mma(d_tmem + mt * BN, sdesc(st + mt * P_BYTES) + 2 * k, qd + 2 * k, IDESC,
                     (i > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(empty(s));
        }
        if (!ok) break;
        tc_commit(tfull(acc));
        ++tile_it;
      }
      // Make sure every issued MMA has finished before TMEM is released.
      tc_commit(final_bar);
      mbar_drain(final_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int q4 = warp & 3;            // TMEM lane quarter this warp may access
    const int row = q4 * 32 + lane;     // accumulator row (P index within a sub-tile)
    uint32_t tile_it = 0;
    SegIter si;
    si.init(p);
    Seg sg;
    while (si.next(p, sg)) {
      const int acc = ACC_BUFS == 2 ? (tile_it & 1) : 0;
      const uint32_t use = ACC_BUFS == 2 ? (tile_it >> 1) : tile_it;
      if (!mbar_wait(tfull(acc), use & 1, abort_flag, 4)) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + ((uint32_t)(q4 * 32) << 16) + acc * ACC_COLS;
      const int q0 = sg.tq * BN;
      if (sg.full) {
#pragma unroll 1
        for (int mt = 0; mt < MT; ++mt) {
          const int pi = (sg.tp * MT + mt) * BM + row;
#pragma unroll 1
          for (int c0 = 0; c0 < BN; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(tacc + mt * BN + c0, r);
            float f[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
            store_chunk(p, pi, q0 + c0, f);
          }
        }
      } else {
        // deposit this partial, then the last of the tile's contributors sums and stores
        constexpr int64_t SLOT = (int64_t)MT * BM * BN;
        float* mine = p.ws + (int64_t)sg.slot * SLOT;
#pragma unroll 1
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll 1
          for (int c0 = 0; c0 < BN; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(tacc + mt * BN + c0, r);
            float4* dst = reinterpret_cast<float4*>(mine + (int64_t)(mt * BM + row) * BN + c0);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              __stcg(dst + j, make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                          __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
          }
        }
        __threadfence();
        __syncwarp();
        int* ctr = p.counters + (int64_t)sg.tile * 4 + q4;
        int prev = 0;
        if (lane == 0) prev = atomicAdd(ctr, 1);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        const int64_t x0 = (int64_t)sg.tile * p.num_kb;
        const int cf = sk_owner(p, x0), cl = sk_owner(p, x0 + p.num_kb - 1);
        if (prev == cl - cf) {
          __threadfence();
#pragma unroll 1
          for (int mt = 0; mt < MT; ++mt) {
            const int pi = (sg.tp * MT + mt) * BM + row;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
              uint32_t r[32];
              tmem_ld32(tacc + mt * BN + c0, r);
              float f[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
              for (int c = cf; c <= cl; ++c) {
                if (c == (int)blockIdx.x) continue;
                const int slot = c * 2 + (sk_start(p, c) < x0 ? 1 : 0);
                const float4* src =
                    reinterpret_cast<const float4*>(p.ws + (int64_t)slot * SLOT + (int64_t)(mt * BM + row) * BN + c0);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const float4 v = __ldcg(src + j);
                  f[4 * j] += v.x;
                  f[4 * j + 1] += v.y;
                  f[4 * j + 2] += v.z;
                  f[4 * j + 3] += v.w;
                }
              }
              store_chunk(p, pi, q0 + c0, f);
            }
          }
          if (lane == 0) *ctr = 0;  // every contributor has arrived: ready for the next launch
        }
      }
      tc_fence_before();
      if (lane == 0) mbar_arrive(tempty(acc));
      ++tile_it;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float4 ld_dsmem_f32x4(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}

// Split-K inside a thread-block cluster (decode-sized problems with few output tiles).
// The `splits` CTAs of a cluster compute disjoint K slices of ONE output tile; each
// exports its fp32 accumulator from TMEM into its own (now idle) stage ring, and after a
// cluster barrier CTA r sums rows [r*128/splits, ...) of all peers' exports through
// distributed shared memory and writes the bf16 result.  No partial sums touch HBM.
// Both cluster barriers are executed unconditionally by every thread (all waits before
// them are bounded), so a CTA that gave up on a wait cannot strand its peers.
template <int BN, int STAGES>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_cluster_kernel(const __grid_constant__ CUtensorMap map_p, const __grid_constant__ CUtensorMap map_q, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int P_BYTES = BM * BK * 2;
  constexpr int Q_BYTES = BN * BK * 2;
  constexpr int STAGE_BYTES = P_BYTES + Q_BYTES;
  constexpr int XLD = BN + 4;  // export row stride in floats (16-byte rows, spread banks)
  static_assert(BM * XLD * 4 <= STAGES * STAGE_BYTES, "export must fit in the stage ring");
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * STAGES + 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 3);
  const uint32_t bar0 = smem_u32(bars);
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
  const uint32_t tfull = bar0 + 8u * (2 * STAGES);
  const uint32_t final_bar = bar0 + 8u * (2 * STAGES + 1);
  float* xp = reinterpret_cast<float*>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;

  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int split = (int)rank;
  int tp, tq, dummy;
  unit_coords(p, blockIdx.x / p.splits, tp, tq, dummy);
  const int kb0 = split * p.kb_per_split, kb1 = min(p.num_kb, kb0 + p.kb_per_split);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(tfull, 1);
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // inputs and the output may belong to the previous kernel in the stream
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_p)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_q)) : "memory");
      uint32_t it = 0;
      bool ok = true;
      const int nkb = kb1 - kb0;
      const int rot = nkb > 0 ? (tp + tq) % nkb : 0;
      const CUtensorMap* wmap = p.swap ? &map_p : &map_q;
      const int wrow = p.swap ? tp * BM : tq * BN;
      if (p.prefetch_w)
        for (int i = 0; i < min(nkb, PF_DIST); ++i) tma_prefetch_2d(wmap, (kb0 + (i + rot) % nkb) * BK, wrow);
      for (int i = 0; i < nkb; ++i, ++it) {
        const int kb = kb0 + (i + rot) % nkb;
        const int s = it % STAGES;
        const uint32_t round = it / STAGES;
        if (p.prefetch_w && i + PF_DIST < nkb) tma_prefetch_2d(wmap, (kb0 + (i + PF_DIST + rot) % nkb) * BK, wrow);
        if (!mbar_wait(empty(s), (round & 1) ^ 1, abort_flag, 5)) {
          ok = false;
          break;
        }
        const uint32_t st = smem_u32(smem + s * STAGE_BYTES);
        mbar_arrive_expect_tx(full(s), STAGE_BYTES);
        tma_load_2d(st, &map_p, full(s), kb * BK, tp * BM);
        tma_load_2d(st + P_BYTES, &map_q, full(s), kb * BK, tq * BN);
      }
      if (!ok) {
        const uint32_t n = it < (uint32_t)STAGES ? it : (uint32_t)STAGES;
        for (uint32_t j = it - n; j < it; ++j) mbar_drain(full(j % STAGES), (j / STAGES) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16<BN>();
      uint32_t it = 0;
      for (int i = 0; i < kb1 - kb0; ++i, ++it) {
        const int s = it % STAGES;
        const uint32_t round = it / STAGES;
        if (!mbar_wait(full(s), round & 1, abort_flag, 6)) break;
        const uint32_t st = smem_u32(smem + s * STAGE_BYTES);
        const uint64_t pd = sdesc(st), qd = sdesc(st + P_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) tc_mma(tmem_base, pd + 2 * k, qd + 2 * k, IDESC, (i > 0 || k > 0) ? 1u : 0u);
        tc_commit(empty(s));
      }
      tc_commit(tfull);
      tc_commit(final_bar);
      mbar_drain(final_bar, 0);
    }
    __syncwarp();
  } else {
    // export the accumulator: row-major [128][BN + 1] fp32 over the idle stage ring
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const bool ok = mbar_wait(tfull, 0, abort_flag, 7);
    tc_fence_after();
    if (ok) {
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(q4 * 32) << 16) + c0, r);
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(xp + row * XLD + c0 + j) =
              make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                          __uint_as_float(r[j + 3]));
      }
    }
    tc_fence_before();
  }
  cluster_sync_all();  // every CTA's export is complete and visible cluster-wide

  const int rows_per = (BM + p.splits - 1) / p.splits;
  const int r0 = split * rows_per, r1 = min(BM, r0 + rows_per);
  const int nrows = r1 - r0;
  constexpr int C4 = BN / 4;
  const int total = nrows > 0 ? nrows * C4 : 0;
  const uint32_t xbase = smem_u32(xp);
  if (p.act && BN >= 32) {
    // 4 output features per item: gates at column g..g+3 of a 32-column group, ups at g+16
    constexpr int O4 = BN / 8;
    for (int idx = threadIdx.x; idx < nrows * O4; idx += NUM_THREADS) {
      const int row = r0 + idx / O4, o4 = idx % O4;
      const int gc = 32 * (o4 >> 2) + 4 * (o4 & 3);
      const int pi = tp * BM + row, qg = tq * BN + gc;
      if (pi >= p.p_rows || qg >= p.q_rows) continue;
      const uint32_t offg = xbase + (uint32_t)(row * XLD + gc) * 4u, offu = offg + 64u;
      float4 vg[8], vu[8];
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2)
        if (s2 < p.splits) {
          vg[s2] = ld_dsmem_f32x4(offg, (uint32_t)s2);
          vu[s2] = ld_dsmem_f32x4(offu, (uint32_t)s2);
        }
      float g[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2)
        if (s2 < p.splits) {
          g[0] += vg[s2].x; g[1] += vg[s2].y; g[2] += vg[s2].z; g[3] += vg[s2].w;
          u[0] += vu[s2].x; u[1] += vu[s2].y; u[2] += vu[s2].z; u[3] += vu[s2].w;
        }
      const float o[4] = {silu_f(g[0]) * u[0], silu_f(g[1]) * u[1], silu_f(g[2]) * u[2], silu_f(g[3]) * u[3]};
      const int oc = (tq * BN + 32 * (o4 >> 2)) / 2 + 4 * (o4 & 3);
      *reinterpret_cast<uint2*>(p.c + (int64_t)pi * p.ldc + oc) = f32_to_bf16x4(o);
    }
  }
  // Each item is 4 consecutive columns of one row; all peers' float4 loads for an item
  // are issued before they are summed.
  for (int idx = p.act ? total : threadIdx.x; idx < total; idx += NUM_THREADS) {
    int row, c4;
    if (p.swap) {  // consecutive threads -> consecutive features (output-contiguous)
      c4 = idx / nrows;
      row = r0 + (idx - c4 * nrows);
    } else {
      row = r0 + idx / C4;
      c4 = idx % C4;
    }
    const int pi = tp * BM + row, qj = tq * BN + c4 * 4;
    if (pi >= p.p_rows || qj >= p.q_rows) continue;
    const uint32_t off = xbase + (uint32_t)(row * XLD + c4 * 4) * 4u;
    float4 v[8];
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2)
      if (s2 < p.splits) v[s2] = ld_dsmem_f32x4(off, (uint32_t)s2);
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2)
      if (s2 < p.splits) {
        a0 += v[s2].x;
        a1 += v[s2].y;
        a2 += v[s2].z;
        a3 += v[s2].w;
      }
    const float f[4] = {a0, a1, a2, a3};
    const int nv = min(4, p.q_rows - qj);
    if (p.swap) {
      for (int e = 0; e < nv; ++e) p.c[(int64_t)(qj + e) * p.ldc + pi] = __float2bfloat16(f[e]);
    } else if (nv == 4) {
      *reinterpret_cast<uint2*>(p.c + (int64_t)pi * p.ldc + qj) = f32_to_bf16x4(f);
    } else {
      for (int e = 0; e < nv; ++e) p.c[(int64_t)pi * p.ldc + qj + e] = __float2bfloat16(f[e]);
    }
  }
  cluster_sync_all();  // peers may still be reading this CTA's export
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool make_map(CUtensorMap* m, const void* base, int rows, int k, int64_t ld_elems, int box_rows,
              CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld_elems * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, int MT = 1>
constexpr int stages_for() {
  return (200 * 1024) / (MT * BM * BK * 2 + BN * BK * 2) > 8 ? 8 : (200 * 1024) / (MT * BM * BK * 2 + BN * BK * 2);
}

template <int BN>
cudaError_t run_cluster(const CUtensorMap& mp, const CUtensorMap& mq, const Params& prm, cudaStream_t stream) {
  constexpr int STAGES = stages_for<BN>();
  constexpr int SMEM = STAGES * (BM * BK * 2 + BN * BK * 2) + 1024 + 256;
  auto kern = gemm_cluster_kernel<BN, STAGES>;
  static std::atomic<uint64_t> done{0};  // per template instance: devices already opted in
  cudaError_t e = smem_opt_in(done, kern, SMEM, /*nonportable_cluster=*/true);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(prm.tiles_p * prm.tiles_q * prm.splits, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = prm.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, mp, mq, prm);
}

template <int BN, int MT = 1>
cudaError_t run(const CUtensorMap& mp, const CUtensorMap& mq, const Params& prm, int grid, cudaStream_t stream) {
  constexpr int STAGES = stages_for<BN, MT>();
  constexpr int SMEM = STAGES * (MT * BM * BK * 2 + BN * BK * 2) + 1024 + 256;
  auto kern = gemm_kernel<BN, STAGES, MT>;
  static std::atomic<uint64_t> done{0};  // per template instance: devices already opted in
  cudaError_t e = smem_opt_in(done, kern, SMEM);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, mp, mq, prm);
}

int num_sms() {
  static std::atomic<int> cached{0};
  int n = cached.load(std::memory_order_relaxed);
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    cached.store(n, std::memory_order_relaxed);
  }
  return n;
}

template <int BN>
int max_active_clusters(int splits) {
  // CTAs of `splits`-wide clusters that can be resident at once (cached per size; atomic entries,
  // so threads that query at the same time only ever store the same value).
  static std::atomic<int> cache[9];
  if (splits < 2 || splits > 8) return 0;
  if (int c = cache[splits].load(std::memory_order_relaxed)) return c;
  constexpr int STAGES = stages_for<BN>();
  constexpr int SMEM = STAGES * (BM * BK * 2 + BN * BK * 2) + 1024 + 256;
  auto kern = gemm_cluster_kernel<BN, STAGES>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits * 64, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM;
  cudaLaunchAttribute attr[2];
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;  // occupancy query: the cluster shape only
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = num_sms() / splits;
  }
  cache[splits].store(n * splits, std::memory_order_relaxed);
  return n * splits;
}

int cluster_capacity(int bn, int splits) {
  switch (bn) {
    case 32: return max_active_clusters<32>(splits);
    case 64: return max_active_clusters<64>(splits);
    case 128: return max_active_clusters<128>(splits);
    default: return max_active_clusters<256>(splits);
  }
}

// Decode-sized GEMM (m <= 256 tokens): every CTA holds ALL token rows (MT sub-tiles of
// 128) against one BN-row slice of the weights, over one K slice; the `splits` K slices of
// a weight slice run as one thread-block cluster and are summed through distributed
// shared memory.  BN (any multiple of 16 up to 256) and splits are runtime values chosen
// so that the clusters fill the GPU in one wave: the weights are then streamed exactly once.
// Streaming the weights from HBM is latency-bound at these sizes, so they get their own
// deep ring (most of shared memory) fed by warp 0, while the activations, which hit in L2,
// get a shallow ring fed by warp 2 (before it turns to the epilogue).
struct DecParams {
  int m, n, k;           // C[m, n] = X[m, k] W[n, k]^T
  int bn, splits, kb_per_split, num_kb;
  int w_stages, a_stages;
  int act;               // 1: SiLU-and-mul epilogue (interleaved gate/up rows, see act_silu_store)
  int a_rows;            // rows of each activation TMA box: m rounded up to 16 when m < 128 (the
                         // accumulator rows past it see stale shared memory and are never stored)
  uint32_t idesc;
  __nv_bfloat16* c;
  int64_t ldc;
  GemmRsEpilogue rs;     // rs.rows > 0: reduce-scatter epilogue (rows stored at their owner rank)
};

// Destination of output row pi: local C, or the owner rank's receive slot for this rank.
__device__ __forceinline__ __nv_bfloat16* dec_row(const DecParams& p, int pi) {
  if (p.rs.rows > 0) {
    const int o = pi / p.rs.rows;
    return static_cast<__nv_bfloat16*>(p.rs.dst[o]) + (int64_t)(pi - o * p.rs.rows) * p.ldc;
  }
  return p.c + (int64_t)pi * p.ldc;
}

// Reduce-scatter arrival (thread 0 of each CTA, after the CTA's stores): the last CTA of the
// grid to arrive publishes this rank's arrival word, the reduction's call number, at every
// rank.  Each CTA's system-scope fence orders its row stores (peer stores included) before
// its arrival on the local counter; the last CTA's acquire of that counter and its own fence
// order all of them before the flag stores.
__device__ __forceinline__ void dec_rs_arrive(const GemmRsEpilogue& rs) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  uint32_t prev;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(rs.ctas_done) : "memory");
  if (prev != gridDim.x * gridDim.y * gridDim.z - 1) return;
  uint32_t calls;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(calls) : "l"(rs.calls) : "memory");
  *rs.ctas_done = 0;  // the next launch that counts starts after this grid completes
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  for (int r = 0; r < rs.world; ++r)
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(rs.flag[r]), "r"(calls + 1) : "memory");
}

template <int MT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_dec_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                    DecParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = MT * BM * BK * 2;
  const int BN = p.bn, SW = p.w_stages, SA = p.a_stages;
  const int W_BYTES = BN * BK * 2;
  const int XLD = BN + 4;  // export row stride in floats
  uint8_t* a_ring = smem;                   // SA x A_BYTES
  uint8_t* w_ring = smem + SA * A_BYTES;    // SW x W_BYTES (1024-aligned: BN % 16 == 0)
  uint64_t* bars = reinterpret_cast<uint64_t*>(w_ring + SW * W_BYTES);
  // bars: wfull[SW], wempty[SW], afull[SA], aempty[SA], tfull, final
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * SW + 2 * SA + 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * SW + 2 * SA + 3);
  const uint32_t bar0 = smem_u32(bars);
  auto wfull = [&](int s) { return bar0 + 8u * s; };
  auto wempty = [&](int s) { return bar0 + 8u * (SW + s); };
  auto afull = [&](int s) { return bar0 + 8u * (2 * SW + s); };
  auto aempty = [&](int s) { return bar0 + 8u * (2 * SW + SA + s); };
  const uint32_t tfull = bar0 + 8u * (2 * SW + 2 * SA);
  const uint32_t final_bar = tfull + 8u;
  float* xp = reinterpret_cast<float*>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // columns read: MT * BN, plus 16 when the last 32-column load of a sub-tile overhangs it
  uint32_t tmem_cols = 32;
  while (tmem_cols < (uint32_t)(MT * BN + (BN % 32 ? 16 : 0))) tmem_cols <<= 1;

  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int split = (int)rank;
  const int tq = blockIdx.x / p.splits;
  const int kb0 = split * p.kb_per_split, kb1 = min(p.num_kb, kb0 + p.kb_per_split);
  const int nkb = kb1 > kb0 ? kb1 - kb0 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SW; ++s) {
      mbar_init(wfull(s), 1);
      mbar_init(wempty(s), 1);
    }
    for (int s = 0; s < SA; ++s) {
      mbar_init(afull(s), 1);
      mbar_init(aempty(s), 1);
    }
    mbar_init(tfull, 1);
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();  // every CTA of this grid is resident (grid <= SMs): let the next kernel launch
  
  if ((warp == 0 || warp == 2) && lane == 0) {
    // ------------------------------------------------ producers: warp 0 weights, warp 2 activations
    const bool is_w = warp == 0;
    const CUtensorMap* map = is_w ? &map_w : &map_x;
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
    const int S = is_w ? SW : SA;
    const uint32_t bytes = is_w ? (uint32_t)W_BYTES : (uint32_t)(MT * p.a_rows * BK * 2);
    // the weights do not depend on the previous kernel: their ring fills while it finishes
    if (!is_w) pdl_wait();
    uint32_t it = 0;
    bool ok = true;
    for (int i = 0; i < nkb; ++i, ++it) {
      const int kb = kb0 + i;
      const int s = it % S;
      const uint32_t round = it / S;
      if (!mbar_wait(is_w ? wempty(s) : aempty(s), (round & 1) ^ 1, abort_flag, 8)) {
        ok = false;
        break;
      }
      const uint32_t fb = is_w ? wfull(s) : afull(s);
      mbar_arrive_expect_tx(fb, bytes);
      if (is_w) {
        tma_load_2d(smem_u32(w_ring + s * W_BYTES), &map_w, fb, kb * BK, tq * BN);
      } else {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          tma_load_2d(smem_u32(a_ring + s * A_BYTES) + mt * (BM * BK * 2), &map_x, fb, kb * BK, mt * BM);
      }
    }
    if (!ok) {
      const uint32_t n = it < (uint32_t)S ? it : (uint32_t)S;
      for (uint32_t j = it - n; j < it; ++j) mbar_drain(is_w ? wfull(j % S) : afull(j % S), (j / S) & 1);
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer
    for (int i = 0; i < nkb; ++i) {
      const int sw = i % SW, sa = i % SA;
      if (!mbar_wait(wfull(sw), (i / SW) & 1, abort_flag, 9)) break;
      if (!mbar_wait(afull(sa), (i / SA) & 1, abort_flag, 9)) break;
      const uint64_t wd = sdesc(smem_u32(w_ring + sw * W_BYTES));
      const uint32_t ab = smem_u32(a_ring + sa * A_BYTES);
#pragma unroll
      for (int k = 0; k < BK / 16; ++k)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          tc_mma(tmem_base + mt * BN, sdesc(ab + mt * (BM * BK * 2)) + 2 * k, wd + 2 * k, p.idesc,
                 (i > 0 || k > 0) ? 1u : 0u);
      tc_commit(wempty(sw));
      tc_commit(aempty(sa));
    }
    tc_commit(tfull);
    tc_commit(final_bar);
    mbar_drain(final_bar, 0);
  }
  __syncwarp();
  bool acc_ok = true;
  if (warp >= 2) {
    acc_ok = (warp == 2 ? mbar_wait : mbar_wait_sleep)(tfull, 0, abort_flag, 10);
    tc_fence_after();
  }
  pdl_wait();  // the output may still be read by the previous kernel in the stream
  pdl_trigger();
  if (p.splits == 1) {
    // whole K in this CTA: accumulator rows straight from TMEM to the output
    if (warp >= 2 && acc_ok) {
      const int q4 = warp & 3;
      const int row = q4 * 32 + lane;
#pragma unroll 1
      for (int mt = 0; mt < MT; ++mt) {
        const int pi = mt * BM + row;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tmem_base + ((uint32_t)(q4 * 32) << 16) + mt * BN + c0, r);
          const int qj = tq * BN + c0;
          const int valid = min(min(32, BN - c0), p.n - qj);
          if (pi >= p.m || valid <= 0) continue;
          float f[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
          if (p.act) {  // bn % 32 == 0 and n % 32 == 0 in this mode
            act_silu_store(dec_row(p, pi) + qj / 2, f);
            continue;
          }
          __nv_bfloat16* dst = dec_row(p, pi) + qj;
          if (valid == 32) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) *reinterpret_cast<uint4*>(dst + j) = f32_to_bf16x8(f + j);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < valid) dst[j] = __float2bfloat16(f[j]);
          }
        }
      }
      tc_fence_before();
    }
    __syncthreads();
  } else {
    const uint32_t xbase = smem_u32(xp);
    const int rows_per = (BM + p.splits - 1) / p.splits;
    const int r0 = split * rows_per, r1 = min(BM, r0 + rows_per);
    const int C4 = BN / 4;
#pragma unroll 1
    for (int mt = 0; mt < MT; ++mt) {
      if (warp >= 2 && acc_ok) {
        // export sub-tile mt: row-major [128][BN + 4] fp32 over the idle rings
        const int q4 = warp & 3;
        const int row = q4 * 32 + lane;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tmem_base + ((uint32_t)(q4 * 32) << 16) + mt * BN + c0, r);
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            if (c0 + j < BN)
              *reinterpret_cast<float4*>(xp + row * XLD + c0 + j) =
                  make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                              __uint_as_float(r[j + 3]));
        }
      }
      if (warp >= 2) tc_fence_before();
      cluster_sync_all();  // every CTA's export of sub-tile mt is visible cluster-wide
      if (p.act) {
        // one row per warp at a time; lane item o4 = 4 output features (gates at column
        // 32 (o4 / 4) + 4 (o4 % 4), ups 16 columns further)
        const int O4 = BN / 8;
#pragma unroll 1
        for (int rr = r0 + warp; rr < r1; rr += NUM_THREADS / 32) {
          const int pi = mt * BM + rr;
          for (int o4 = lane; o4 < O4; o4 += 32) {
            const int gc = 32 * (o4 >> 2) + 4 * (o4 & 3);
            const uint32_t offg = xbase + (uint32_t)(rr * XLD + gc) * 4u, offu = offg + 64u;
            float4 vg[8], vu[8];
#pragma unroll
            for (int s2 = 0; s2 < 8; ++s2)
              if (s2 < p.splits) {
                vg[s2] = ld_dsmem_f32x4(offg, (uint32_t)s2);
                vu[s2] = ld_dsmem_f32x4(offu, (uint32_t)s2);
              }
            float g[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int s2 = 0; s2 < 8; ++s2)
              if (s2 < p.splits) {
                g[0] += vg[s2].x; g[1] += vg[s2].y; g[2] += vg[s2].z; g[3] += vg[s2].w;
                u[0] += vu[s2].x; u[1] += vu[s2].y; u[2] += vu[s2].z; u[3] += vu[s2].w;
              }
            const int qg = tq * BN + gc;
            if (pi >= p.m || qg >= p.n) continue;
            const float o[4] = {silu_f(g[0]) * u[0], silu_f(g[1]) * u[1], silu_f(g[2]) * u[2],
                                silu_f(g[3]) * u[3]};
            const int oc = (tq * BN + 32 * (o4 >> 2)) / 2 + 4 * (o4 & 3);
            *reinterpret_cast<uint2*>(dec_row(p, pi) + oc) = f32_to_bf16x4(o);
          }
        }
      }
      // one row per warp at a time, lanes along the columns (coalesced DSMEM reads and
      // stores); two rows in flight per warp
#pragma unroll 1
      for (int rr = p.act ? r1 : r0 + warp; rr < r1; rr += 2 * (NUM_THREADS / 32)) {
        const int rr2 = rr + NUM_THREADS / 32;
        const bool has2 = rr2 < r1;
        const int pi = mt * BM + rr, pi2 = mt * BM + rr2;
        for (int c4 = lane; c4 < C4; c4 += 32) {
          const int qj = tq * BN + c4 * 4;
          const uint32_t off = xbase + (uint32_t)(rr * XLD + c4 * 4) * 4u;
          const uint32_t off2 = xbase + (uint32_t)(rr2 * XLD + c4 * 4) * 4u;
          float4 v[8], v2[8];
#pragma unroll
          for (int s2 = 0; s2 < 8; ++s2)
            if (s2 < p.splits) {
              v[s2] = ld_dsmem_f32x4(off, (uint32_t)s2);
              if (has2) v2[s2] = ld_dsmem_f32x4(off2, (uint32_t)s2);
            }
          float f[4] = {0.f, 0.f, 0.f, 0.f}, g[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int s2 = 0; s2 < 8; ++s2)
            if (s2 < p.splits) {
              f[0] += v[s2].x;
              f[1] += v[s2].y;
              f[2] += v[s2].z;
              f[3] += v[s2].w;
              if (has2) {
                g[0] += v2[s2].x;
                g[1] += v2[s2].y;
                g[2] += v2[s2].z;
                g[3] += v2[s2].w;
              }
            }
          if (qj >= p.n) continue;
          const int nv = min(4, p.n - qj);
          if (pi < p.m) {
            if (nv == 4) *reinterpret_cast<uint2*>(dec_row(p, pi) + qj) = f32_to_bf16x4(f);
            else
              for (int e = 0; e < nv; ++e) dec_row(p, pi)[qj + e] = __float2bfloat16(f[e]);
          }
          if (has2 && pi2 < p.m) {
            if (nv == 4) *reinterpret_cast<uint2*>(dec_row(p, pi2) + qj) = f32_to_bf16x4(g);
            else
              for (int e = 0; e < nv; ++e) dec_row(p, pi2)[qj + e] = __float2bfloat16(g[e]);
          }
        }
      }
      cluster_sync_all();  // peers may still be reading this CTA's export
    }
  }
  if (p.rs.rows > 0) {
    __syncthreads();  // every row store of this CTA is issued
    if (threadIdx.x == 0) dec_rs_arrive(p.rs);
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols));
  }
}

constexpr int DEC_SMEM_MAX = 232448;  // opt-in dynamic shared memory per block on sm_100

struct DecCfg {
  int mt, bn, splits, kb_per_split, w_stages, a_stages, smem, tiles;
  double cost;
  double traffic = 0.0;  // waves x bytes one CTA moves through its shared memory (see dec_candidates)
};

template <int MT>
int dec_capacity(int splits, int smem) {
  // CTAs of `splits`-wide clusters of this shape that can be resident at once
  static std::map<std::pair<int, int>, int> cache;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  auto key = std::make_pair(splits, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  auto kern = gemm_dec_kernel<MT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DEC_SMEM_MAX);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits * 64, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[2];
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;  // occupancy query: the cluster shape only
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = num_sms() / splits;
  }
  cache[key] = n * splits;
  return n * splits;
}

// All decode-kernel shapes for C[m, n] (m <= 256), cheapest first by a bytes-per-CTA model:
// waves x (weight + activation bytes one CTA streams + its share of the reduction + a fixed
// pipeline-fill cost).  `traffic` is a second ranking: waves x (bytes one CTA loads into shared
// memory: its weight slice AND all m activation rows of its K range, plus the fp32 partial it
// exports and reads back in a split-K reduction).  At m >= 128 the activation rows, re-read by
// every CTA, outweigh the weights unless the slice is wide, which the first model ignores.
std::vector<DecCfg> dec_candidates(int m, int n, int k, bool by_traffic = false) {
  std::vector<DecCfg> out;
  if (m <= 0 || m > 2 * BM || k % BK) return out;
  const int mt = m > BM ? 2 : 1;
  const int num_kb = k / BK;
  const int a_bytes = mt * BM * BK * 2;
  for (int a_st : {3, 4}) {
    for (int bn = 32; bn <= 256; bn += 16) {
      const int w_bytes = bn * BK * 2;
      const int fixed = 1024 + a_st * a_bytes + 512;
      int w_st = (DEC_SMEM_MAX - fixed) / w_bytes;
      if (w_st > 12) w_st = 12;
      if (w_st < 2 || 512 * (bn + 4) > a_st * a_bytes + w_st * w_bytes) continue;
      const int smem = fixed + w_st * w_bytes;
      const int tiles = (n + bn - 1) / bn;
      int prev = 0;
      for (int sp = 1; sp <= 8; ++sp) {
        const int kbs = (num_kb + sp - 1) / sp;
        const int s_eff = (num_kb + kbs - 1) / kbs;
        if (s_eff == prev) continue;
        prev = s_eff;
        const int cap = mt == 2 ? dec_capacity<2>(s_eff, smem) : dec_capacity<1>(s_eff, smem);
        const int units = tiles * s_eff;
        const int waves = (units + cap - 1) / (cap > 0 ? cap : 1);
        // time ~ waves x (weight bytes of one CTA / bytes it keeps in flight) x latency, plus
        // the reduction and a fixed start-up cost, in units of one latency
        const double w_cta = (double)kbs * w_bytes;
        const double inflight = (double)(w_st < kbs ? w_st : kbs) * w_bytes;
        const double red = s_eff > 1 ? 0.5 * mt * BM * bn * 4 / 65536.0 : 0.0;
        DecCfg c{mt, bn, s_eff, kbs, w_st, a_st, smem, tiles, waves * (w_cta / inflight + red + 2.0)};
        const double red_bytes = s_eff > 1 ? 2.0 * mt * BM * bn * 4 : 0.0;
        c.traffic = waves * ((double)kbs * (w_bytes + a_bytes) + red_bytes);
        out.push_back(c);
      }
    }
  }
  if (by_traffic)
    std::sort(out.begin(), out.end(), [](const DecCfg& a, const DecCfg& b) { return a.traffic < b.traffic; });
  else
    std::sort(out.begin(), out.end(), [](const DecCfg& a, const DecCfg& b) { return a.cost < b.cost; });
  return out;
}

cudaError_t run_dec(const DecCfg& d, const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc,
                    int m, int n, int k, cudaStream_t stream, int act = 0, const GemmRsEpilogue* rs = nullptr) {
  if (act && (d.bn % 32 || n % 32)) return cudaErrorInvalidValue;
  CUtensorMap mx, mw;
  const int a_rows = d.mt == 1 && m < BM ? ((m + 15) / 16) * 16 : BM;
  if (!make_map(&mx, x, m, k, ldx, a_rows) || !make_map(&mw, w, n, k, ldw, d.bn)) return cudaErrorInvalidValue;
  DecParams p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.bn = d.bn;
  p.splits = d.splits;
  p.kb_per_split = d.kb_per_split;
  p.num_kb = k / BK;
  p.w_stages = d.w_stages;
  p.act = act;
  p.a_rows = a_rows;
  p.a_stages = d.a_stages;
  p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(d.bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
  p.c = static_cast<__nv_bfloat16*>(c);
  p.ldc = ldc;
  if (rs) {
    if (act || rs->rows <= 0 || rs->world < 1 || rs->world > 8 || !rs->calls || !rs->ctas_done ||
        (int64_t)rs->rows * rs->world < m || ldc % 8)
      return cudaErrorInvalidValue;
    for (int r = 0; r < rs->world; ++r)
      if (!rs->dst[r] || !rs->flag[r] || ((uintptr_t)rs->dst[r] & 15)) return cudaErrorInvalidValue;
    p.rs = *rs;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(d.tiles * d.splits, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = d.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = d.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  static std::atomic<uint64_t> done[3];  // devices already opted in, per MMA row-tile count
  if (d.mt == 2) {
    cudaError_t e = smem_opt_in(done[2], gemm_dec_kernel<2>, DEC_SMEM_MAX);
    if (e != cudaSuccess) return e;
    return cudaLaunchKernelEx(&cfg, gemm_dec_kernel<2>, mx, mw, p);
  }
  cudaError_t e = smem_opt_in(done[1], gemm_dec_kernel<1>, DEC_SMEM_MAX);
  if (e != cudaSuccess) return e;
  return cudaLaunchKernelEx(&cfg, gemm_dec_kernel<1>, mx, mw, p);
}


// ------------------------------------------------------------------ CTA-pair decode GEMM
// C[m, n] = X[m, k] W[n, k]^T for 128 < m <= 256 tokens with one M = 256 MMA per k-step over a
// pair of CTAs (tcgen05.mma.cta_group::2, issued by the even CTA of a 2-CTA cluster).  Each CTA
// of the pair stages its own 128 token rows and HALF of the pair's BN weight rows, so per pair a
// weight byte and an activation row each cross into shared memory once: against one CTA that
// holds all 256 tokens, a CTA moves half the activation bytes, which is what bounds the decode
// kernel at these sizes (the activations come from L2 once per CTA).  Both CTAs' TMA loads
// complete on the even CTA's stage barrier (unicast loads; the barrier address is mapped into the
// even CTA with mapa); the even CTA's commits arrive on both CTAs' barriers (commit multicast).
// Each CTA's TMEM holds the fp32 accumulator of its 128 tokens x BN outputs; warps 2-5 of both
// CTAs store it (optionally SiLU-and-mul of interleaved gate/up rows).  Warps: 0 TMA, 1 TMEM +
// MMA (even CTA), 2-5 epilogue.
struct PairParams {
  int m, n, k, bn, num_kb, stages, act;
  uint32_t idesc;
  __nv_bfloat16* c;
  int64_t ldc;
};

__device__ __forceinline__ uint32_t cluster_map(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}

// Unicast TMA load into this CTA's shared memory that completes on a barrier of either CTA of
// the pair (here always the even CTA's).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Arrive on the barrier at this shared-memory offset in every CTA of `mask` once the pair's
// MMAs issued so far have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                     PairParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = BM * BK * 2;  // this CTA's 128 token rows of one k-block
  const int HB = p.bn / 2;              // weight rows staged by this CTA
  const int W_BYTES = HB * BK * 2;
  const int STAGE = A_BYTES + W_BYTES;  // HB % 8 == 0: every tile stays 1024-aligned
  const int S = p.stages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * STAGE);
  // bars: full[S] (used in the even CTA), empty[S], tfull, final
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * S + 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 3);
  const uint32_t bar0 = smem_u32(bars);
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (S + s); };
  const uint32_t tfull = bar0 + 8u * (2 * S);
  const uint32_t final_bar = tfull + 8u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t tmem_cols = 32;
  while (tmem_cols < (uint32_t)p.bn) tmem_cols <<= 1;
  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(tfull, 1);
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {  // the same warp in both CTAs: one allocation that spans the pair
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before any load or commit reaches them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------------ producer (both CTAs)
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_w)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_x)) : "memory");
    const int wrow = pair * p.bn + (int)rank * HB;
    auto kb_of = [&](int i) { return i; };
    const int pre = p.num_kb < S ? p.num_kb : S;
    for (int i = 0; i < pre; ++i) {  // weights first: independent of the previous kernel
      if (leader) mbar_arrive_expect_tx(full(i), 2u * (uint32_t)STAGE);
      tma_load_2d_pair(smem_u32(smem + i * STAGE + A_BYTES), &map_w, cluster_map(full(i), 0), kb_of(i) * BK, wrow);
    }
    pdl_wait();  // the activations come from the previous kernel
    for (int i = 0; i < pre; ++i)
      tma_load_2d_pair(smem_u32(smem + i * STAGE), &map_x, cluster_map(full(i), 0), kb_of(i) * BK, (int)rank * BM);
    bool ok = true;
    int it = pre;
    for (int i = pre; i < p.num_kb; ++i, ++it) {
      const int s = i % S;
      if (!mbar_wait(empty(s), ((i / S) & 1) ^ 1, abort_flag, 30)) {
        ok = false;
        break;
      }
      if (leader) mbar_arrive_expect_tx(full(s), 2u * (uint32_t)STAGE);
      const uint32_t fb = cluster_map(full(s), 0);
      tma_load_2d_pair(smem_u32(smem + s * STAGE + A_BYTES), &map_w, fb, kb_of(i) * BK, wrow);
      tma_load_2d_pair(smem_u32(smem + s * STAGE), &map_x, fb, kb_of(i) * BK, (int)rank * BM);
    }
    if (!ok && leader) {
      const int n = it < S ? it : S;
      for (int j = it - n; j < it; ++j) mbar_drain(full(j % S), (j / S) & 1);
    }
  } else if (warp == 1 && leader) {
    // ------------------------------------------------------------------ MMA issuer (even CTA)
    // converged warp, one elected lane issues; the TMEM base is broadcast so it is warp-uniform
    const uint32_t tbase = __shfl_sync(0xffffffffu, tmem_base, 0);
    for (int i = 0; i < p.num_kb; ++i) {
      const int s = i % S;
      int okw = 1;
      if (lane == 0) okw = mbar_wait(full(s), (i / S) & 1, abort_flag, 31);
      okw = __shfl_sync(0xffffffffu, okw, 0);
      if (!okw) break;
      const uint32_t st = smem_u32(smem + s * STAGE);
      const uint64_t ad = sdesc(st), wd = sdesc(st + A_BYTES);
      if (elect_one()) {
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) tc_mma_pair(tbase, ad + 2 * k, wd + 2 * k, p.idesc, (i > 0 || k > 0) ? 1u : 0u);
        tc_commit_pair(empty(s), 0x3);
      }
      __syncwarp();
    }
    if (elect_one()) {
      tc_commit_pair(tfull, 0x3);
      tc_commit_pair(final_bar, 0x1);
      mbar_drain(final_bar, 0);  // every MMA of the pair has completed before this warp goes on
    }
    __syncwarp();
  }
  __syncwarp();
  if (warp >= 2) {
    const bool acc_ok = (warp == 2 ? mbar_wait : mbar_wait_sleep)(tfull, 0, abort_flag, 32);
    tc_fence_after();
    pdl_wait();  // C may still be read by the previous kernel in the stream
    const int q4 = warp & 3;
    const int row = (int)rank * BM + q4 * 32 + lane;  // token of this thread
#pragma unroll 1
    for (int c0 = 0; c0 < p.bn; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tmem_base + ((uint32_t)(q4 * 32) << 16) + c0, r);
      float f[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
      const int qj = pair * p.bn + c0;
      const int valid = min(32, p.n - qj);
      if (!acc_ok || row >= p.m || valid <= 0) continue;
      __nv_bfloat16* crow = p.c + (int64_t)row * p.ldc;
      if (p.act) {  // bn % 32 == 0 and n % 32 == 0 in this mode
        act_silu_store(crow + qj / 2, f);
        continue;
      }
      __nv_bfloat16* dst = crow + qj;
      if (valid == 32) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) *reinterpret_cast<uint4*>(dst + j) = f32_to_bf16x8(f + j);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < valid) dst[j] = __float2bfloat16(f[j]);
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  cluster_sync_all();  // the pair's MMAs, loads and commits are all done before TMEM is freed
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols));
  }
}

struct PairCfg {
  int bn, stages, smem, pairs;
};

static int pair_smem(int bn, int stages) { return 1024 + stages * (BM * BK * 2 + bn / 2 * BK * 2) + 8 * (2 * stages + 6); }

static int pair_capacity(int smem) {
  // CTAs of 2-CTA clusters with this shared memory that can be resident at once (cached)
  static std::map<int, int> cache;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(smem);
  if (it != cache.end()) return it->second;
  cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DEC_SMEM_MAX);
  cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 64, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = num_sms() / 2;
  }
  cache[smem] = 2 * n;
  return 2 * n;
}

// Pair-kernel configurations for 128 < m <= 256: BN (the pair's weight rows, a multiple of 32) and
// the ring depth, fewest (waves x bytes per CTA) first.
std::vector<PairCfg> pair_candidates(int m, int n, int k, int act) {
  std::vector<PairCfg> out;
  if (m <= BM || m > 2 * BM || k % BK || (act && n % 32)) return out;
  const int num_kb = k / BK;
  std::vector<std::pair<double, PairCfg>> scored;
  for (int bn = 32; bn <= 256; bn += 32) {
    const int pairs = (n + bn - 1) / bn;
    const int stage = BM * BK * 2 + bn / 2 * BK * 2;
    for (int two = 0; two < 2; ++two) {  // one or two CTAs per SM
      const int budget = two ? DEC_SMEM_MAX / 2 - 2048 : DEC_SMEM_MAX;
      int st = (budget - 1024 - 8 * 32) / stage;
      if (st > 10) st = 10;
      if (st > num_kb) st = num_kb;
      if (st < 2) continue;
      const int smem = pair_smem(bn, st);
      if (smem > budget) continue;
      const int cap = pair_capacity(smem);
      const int waves = (2 * pairs + cap - 1) / (cap > 0 ? cap : 1);
      if (waves > 4) continue;
      scored.push_back({(double)waves * num_kb * stage, PairCfg{bn, st, smem, pairs}});
    }
  }
  std::sort(scored.begin(), scored.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
  for (auto& s : scored) out.push_back(s.second);
  return out;
}

cudaError_t run_pair(const PairCfg& d, const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc,
                     int m, int n, int k, cudaStream_t stream, int act = 0) {
  if (m <= BM || m > 2 * BM || k % BK || d.bn % 32 || d.bn > 256 || (act && n % 32) || ldc % 8 || !c ||
      ((uintptr_t)c & 15))
    return cudaErrorInvalidValue;
  CUtensorMap mx, mw;
  if (!make_map(&mx, x, m, k, ldx, BM) || !make_map(&mw, w, n, k, ldw, d.bn / 2)) return cudaErrorInvalidValue;
  PairParams p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.bn = d.bn;
  p.num_kb = k / BK;
  p.stages = d.stages;
  p.act = act;
  // D f32, A bf16 (tokens), B bf16 (weights), N = bn, M = 256 over the pair
  p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(d.bn >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
  p.c = static_cast<__nv_bfloat16*>(c);
  p.ldc = ldc;
  static std::atomic<uint64_t> done{0};
  cudaError_t e = smem_opt_in(done, gemm_pair_kernel, DEC_SMEM_MAX);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * d.pairs, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = d.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, gemm_pair_kernel, mx, mw, p);
}

// ------------------------------------------------------------------ skinny decode GEMM
// Decode-sized GEMM with the WEIGHTS on the MMA's M side (tensor-core "swap" form):
// D[i, j] = sum_k W[i, k] X[j, k] on tiles of MW x 128 weight rows (one M = 128 MMA each)
// by NP tokens (the MMA's N: m rounded up to a multiple of 16, <= 256), so a 1-token step
// moves 16 activation rows per k-block instead of 128 and every shared-memory byte but
// those few is a weight byte.  The K range of a tile is split over the `splits` CTAs of a
// thread-block cluster; every CTA exports its fp32 accumulator transposed ([token][feature])
// into its idle stage ring and, after a cluster barrier, CTA r sums its share of the
// features over the peers through distributed shared memory and stores whole 16-byte runs
// of C rows (optionally SiLU-and-mul of interleaved gate/up rows, or the tensor-parallel
// reduce-scatter destinations of GemmRsEpilogue).  Warps: 0 TMA (weights are loaded before
// griddepcontrol.wait: they do not depend on the previous kernel), 1 TMEM + MMA, 2-5
// TMEM export; all six warps reduce and store.
struct SkParams {
  int m, n, k;
  int np;            // MMA N (tokens per tile, multiple of 16)
  int mrows;         // MMA M: weight rows per sub-tile (128, or 64: twice the CTAs without split-K)
  int mw;            // weight sub-tiles per CTA (1 or 2; 1 when mrows = 64)
  int splits, kb_per_split, num_kb, stages;
  int act;           // 1: SiLU-and-mul epilogue (gate/up rows interleaved in groups of 16)
  int blocked;       // 1: W stored as [n / 128][k / 64][128][64] (every TMA box one contiguous 16 KB)
  uint64_t* trace;   // optional: per CTA SK_TRACE %globaltimer stamps (start, weights issued, first stage
                     // full, MMAs done, export done, reduce done, end, unused; then per k-block times)
  uint32_t idesc;
  __nv_bfloat16* c;
  int64_t ldc;
  GemmRsEpilogue rs;
};

// Trace words per CTA: 8 phase stamps, then the issue time of k-blocks S..63 (index 8 + i; the
// first S are issued before the loop, at stamp 1), the time the MMA thread saw k-blocks 0..63
// land (index 72 + i), the time it started waiting for them (index 136 + i), the time its MMAs
// for them were issued (index 200 + i) and the time its commits were issued (index 264 + i).
constexpr int SK_TRACE = 328;

// TMA coordinates of the weight box (128 rows from `row`, k-block kb).
__device__ __forceinline__ void sk_wcoord(const SkParams& p, int row, int kb, int& x, int& y) {
  if (p.blocked) {
    x = 0;
    y = ((row / BM) * p.num_kb + kb) * BM;
  } else {
    x = kb * BK;
    y = row;
  }
}

__device__ __forceinline__ __nv_bfloat16* sk_row(const SkParams& p, int j) {
  if (p.rs.rows > 0) {
    const int o = j / p.rs.rows;
    return static_cast<__nv_bfloat16*>(p.rs.dst[o]) + (int64_t)(j - o * p.rs.rows) * p.ldc;
  }
  return p.c + (int64_t)j * p.ldc;
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

constexpr int SK_XLD = BM + 4;  // export row stride (floats): [token][128 features + pad]

__global__ void __launch_bounds__(NUM_THREADS, 2)  // two CTAs per SM when their rings fit
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                       SkParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int MR = p.mrows;
  const int W_BYTES = p.mw * MR * BK * 2;
  const int X_BYTES = p.np * BK * 2;
  const int STAGE = W_BYTES + X_BYTES;  // multiple of 2 KB: every operand tile stays 1024-aligned
  const int S = p.stages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * STAGE);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * S + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 2);
  const uint32_t bar0 = smem_u32(bars);
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (S + s); };
  const uint32_t tfull = bar0 + 8u * (2 * S);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t tmem_cols = 32;
  while (tmem_cols < (uint32_t)(p.mw * p.np)) tmem_cols <<= 1;

  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int split = (int)rank;
  const int tq = blockIdx.x / p.splits;
  const int kb0 = split * p.kb_per_split, kb1 = min(p.num_kb, kb0 + p.kb_per_split);
  const int nkb = kb1 > kb0 ? kb1 - kb0 : 0;
  const int wrow0 = tq * p.mw * MR;  // first weight row (output feature) of this tile
  auto kb_of = [&](int i) { return kb0 + i; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(tfull, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();  // the whole grid is resident (one wave): the next kernel may launch
  uint64_t* tr = p.trace ? p.trace + (int64_t)blockIdx.x * SK_TRACE : nullptr;
  if (tr && threadIdx.x == 0) tr[0] = globaltimer();

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------------ producer
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_w)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_x)) : "memory");
    const int pre = nkb < S ? nkb : S;
    for (int i = 0; i < pre; ++i) {  // weights first: independent of the previous kernel
      const int kb = kb_of(i);
      mbar_arrive_expect_tx(full(i), (uint32_t)STAGE);
      for (int w = 0; w < p.mw; ++w) {
        int wx, wy;
        sk_wcoord(p, wrow0 + w * MR, kb, wx, wy);
        tma_load_2d(smem_u32(smem + i * STAGE + w * MR * BK * 2), &map_w, full(i), wx, wy);
      }
    }
    if (tr) tr[1] = globaltimer();
    pdl_wait();  // the activations come from the previous kernel
    for (int i = 0; i < pre; ++i) tma_load_2d(smem_u32(smem + i * STAGE + W_BYTES), &map_x, full(i), kb_of(i) * BK, 0);
    bool ok = true;
    uint32_t it = pre;
    for (int i = pre; i < nkb; ++i, ++it) {
      const int s = i % S;
      if (!mbar_wait(empty(s), ((i / S) & 1) ^ 1, abort_flag, 20)) {
        ok = false;
        break;
      }
      const int kb = kb_of(i);
      if (tr && i < 64) tr[8 + i] = globaltimer();
      mbar_arrive_expect_tx(full(s), (uint32_t)STAGE);
      for (int w = 0; w < p.mw; ++w) {
        int wx, wy;
        sk_wcoord(p, wrow0 + w * MR, kb, wx, wy);
        tma_load_2d(smem_u32(smem + s * STAGE + w * MR * BK * 2), &map_w, full(s), wx, wy);
      }
      tma_load_2d(smem_u32(smem + s * STAGE + W_BYTES), &map_x, full(s), kb * BK, 0);
    }
    if (!ok) {
      const uint32_t n = it < (uint32_t)S ? it : (uint32_t)S;
      for (uint32_t j = it - n; j < it; ++j) mbar_drain(full(j % S), (j / S) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop and one elected lane issues (about 8% faster per stage than
    // a lone lane running it); the TMEM base is broadcast so it is provably warp-uniform.
    const uint32_t tbase = __shfl_sync(0xffffffffu, tmem_base, 0);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % S;
      if (tr && lane == 0 && i < 64) tr[136 + i] = globaltimer();
      int okw = 1;
      if (lane == 0) okw = mbar_wait(full(s), (i / S) & 1, abort_flag, 21);
      okw = __shfl_sync(0xffffffffu, okw, 0);
      if (!okw) break;
      if (tr && lane == 0 && i == 0) tr[2] = globaltimer();
      if (tr && lane == 0 && i < 64) tr[72 + i] = globaltimer();
      const uint32_t st = smem_u32(smem + s * STAGE);
      const uint64_t xd = sdesc(st + W_BYTES);
      if (elect_one()) {
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          for (int w = 0; w < p.mw; ++w)
            tc_mma(tbase + w * p.np, sdesc(st + w * MR * BK * 2) + 2 * k, xd + 2 * k, p.idesc,
                   (i > 0 || k > 0) ? 1u : 0u);
        if (tr && i < 64) tr[200 + i] = globaltimer();
        tc_commit(empty(s));
        if (tr && i < 64) tr[264 + i] = globaltimer();
      }
      __syncwarp();
    }
    if (elect_one()) tc_commit(tfull);
  }
  __syncwarp();
  bool acc_ok = true;
  if (warp >= 2) {
    acc_ok = (warp == 2 ? mbar_wait : mbar_wait_sleep)(tfull, 0, abort_flag, 22);
    tc_fence_after();
    if (tr && threadIdx.x == 64) tr[3] = globaltimer();
  }
  pdl_wait();  // C (or a peer's receive slot) may still be read by the previous kernel
  float* xp0 = reinterpret_cast<float*>(smem);  // export [sub-tile][token][SK_XLD] over the idle ring
  const int fpr = ((MR / p.splits + 7) / 8) * 8;  // features per CTA in the reduction (multiple of 8)
  const int f0 = split * fpr, f1 = min(MR, f0 + fpr);
  // every sub-tile's export at once when the ring holds them all (one pair of cluster barriers),
  // otherwise one sub-tile at a time
  const int per_pass = (int64_t)p.mw * p.np * SK_XLD * 4 <= (int64_t)S * STAGE ? p.mw : 1;
  for (int w0 = 0; w0 < p.mw; w0 += per_pass) {
    if (warp >= 2 && acc_ok) {
      const int q4 = warp & 3;
      // feature row of this thread inside a sub-tile: M = 128 fills every TMEM lane; M = 64 puts
      // rows 16 q .. 16 q + 15 in lanes 32 q .. 32 q + 15 of each warp's quarter
      const int r = MR == BM ? q4 * 32 + lane : q4 * 16 + lane;
      const bool live = MR == BM || lane < 16;
      for (int w = w0; w < w0 + per_pass; ++w) {
        float* xp = xp0 + (w - w0) * p.np * SK_XLD;
        for (int c0 = 0; c0 < p.np; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(tmem_base + ((uint32_t)(q4 * 32) << 16) + w * p.np + c0, v);
          if (live) {
#pragma unroll
            for (int e = 0; e < 16; ++e) xp[(c0 + e) * SK_XLD + r] = __uint_as_float(v[e]);
          }
        }
      }
    }
    if (warp >= 2) tc_fence_before();
    cluster_sync_all();  // every CTA's export of these sub-tiles is visible cluster-wide
    if (tr && threadIdx.x == 0 && w0 == 0) tr[4] = globaltimer();
    for (int w = w0; w < w0 + per_pass; ++w) {
      const uint32_t xbase = smem_u32(xp0 + (w - w0) * p.np * SK_XLD);
      const int fbase = wrow0 + w * MR;  // output feature of row 0 of this sub-tile
      if (p.act) {
        // outputs: 16 per 32 rows (rows 32g..32g+15 gates, +16 the ups); items = 8 outputs
        const int g0 = f0 / 32, g1 = (f1 + 31) / 32;
        const int per_tok = (g1 - g0) * 2;
        for (int it = threadIdx.x; it < p.m * per_tok; it += NUM_THREADS) {
          const int j = it / per_tok, q = it % per_tok;
          const int g = g0 + q / 2, half = q % 2;
          const int rg = g * 32 + half * 8;  // gate rows rg..rg+7, up rows rg+16..rg+23
          if (rg < f0 || rg >= f1 || fbase + rg >= p.n) continue;
          float gv[8] = {0, 0, 0, 0, 0, 0, 0, 0}, uv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
          const uint32_t a = xbase + (uint32_t)(j * SK_XLD + rg) * 4u;
#pragma unroll
          for (int sb = 0; sb < 8; sb += 4) {  // 4 peers' loads in flight at a time
            float4 x0[4], x1[4], y0[4], y1[4];
#pragma unroll
            for (int q = 0; q < 4; ++q)
              if (sb + q < p.splits) {
                x0[q] = ld_dsmem_f32x4(a, sb + q);
                x1[q] = ld_dsmem_f32x4(a + 16u, sb + q);
                y0[q] = ld_dsmem_f32x4(a + 64u, sb + q);
                y1[q] = ld_dsmem_f32x4(a + 80u, sb + q);
              }
#pragma unroll
            for (int q = 0; q < 4; ++q)
              if (sb + q < p.splits) {
                gv[0] += x0[q].x; gv[1] += x0[q].y; gv[2] += x0[q].z; gv[3] += x0[q].w;
                gv[4] += x1[q].x; gv[5] += x1[q].y; gv[6] += x1[q].z; gv[7] += x1[q].w;
                uv[0] += y0[q].x; uv[1] += y0[q].y; uv[2] += y0[q].z; uv[3] += y0[q].w;
                uv[4] += y1[q].x; uv[5] += y1[q].y; uv[6] += y1[q].z; uv[7] += y1[q].w;
              }
          }
          float o[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = silu_f(gv[e]) * uv[e];
          const int oc = (fbase + g * 32) / 2 + half * 8;
          *reinterpret_cast<uint4*>(sk_row(p, j) + oc) = f32_to_bf16x8(o);
        }
      } else {
        const int per_tok = (f1 - f0 + 7) / 8;
        for (int it = threadIdx.x; it < p.m * per_tok; it += NUM_THREADS) {
          const int j = it / per_tok, f = f0 + (it % per_tok) * 8;
          const int feat = fbase + f;
          if (f >= f1 || feat >= p.n) continue;
          float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
          const uint32_t a = xbase + (uint32_t)(j * SK_XLD + f) * 4u;
          float4 x0[8], x1[8];
#pragma unroll
          for (int s2 = 0; s2 < 8; ++s2)  // every peer's loads in flight before the first is used
            if (s2 < p.splits) {
              x0[s2] = ld_dsmem_f32x4(a, s2);
              x1[s2] = ld_dsmem_f32x4(a + 16u, s2);
            }
#pragma unroll
          for (int s2 = 0; s2 < 8; ++s2)
            if (s2 < p.splits) {
              acc[0] += x0[s2].x; acc[1] += x0[s2].y; acc[2] += x0[s2].z; acc[3] += x0[s2].w;
              acc[4] += x1[s2].x; acc[5] += x1[s2].y; acc[6] += x1[s2].z; acc[7] += x1[s2].w;
            }
          __nv_bfloat16* dst = sk_row(p, j) + feat;
          if (feat + 8 <= p.n) {
            *reinterpret_cast<uint4*>(dst) = f32_to_bf16x8(acc);
          } else {
            for (int e = 0; e < 8 && feat + e < p.n; ++e) dst[e] = __float2bfloat16(acc[e]);
          }
        }
      }
    }
    cluster_sync_all();  // peers are done reading this CTA's export before it is overwritten / freed
    if (tr && threadIdx.x == 0 && w0 == 0) tr[5] = globaltimer();
  }
  if (p.rs.rows > 0) {
    __syncthreads();
    if (threadIdx.x == 0) dec_rs_arrive(p.rs);
  }
  if (tr && threadIdx.x == 0) tr[6] = globaltimer();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols));
  }
}

struct SkCfg {
  int np, mw, splits, kb_per_split, stages, smem, tiles;
  int mrows = BM;  // weight rows per MMA (128 or 64)
};

int sk_smem(int np, int mw, int stages, int mrows = BM) {
  const int stage = mw * mrows * BK * 2 + np * BK * 2;
  const int ring = stages * stage;
  const int exportb = np * SK_XLD * 4;
  return 1024 + (ring > exportb ? ring : exportb) + 8 * (2 * stages + 4);
}

int sk_capacity(int splits, int smem) {
  // CTAs of `splits`-wide clusters of this shape that can be resident at once (cached)
  static std::map<std::pair<int, int>, int> cache;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  auto key = std::make_pair(splits, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  cudaFuncSetAttribute(gemm_skinny_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DEC_SMEM_MAX);
  if (splits == 1) {  // no cluster: CTAs per SM x SMs
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemm_skinny_kernel, NUM_THREADS, smem) != cudaSuccess ||
        per_sm <= 0) {
      cudaGetLastError();
      per_sm = 1;
    }
    cache[key] = per_sm * num_sms();
    return cache[key];
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits * 64, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_skinny_kernel, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = num_sms() / splits;
  }
  cache[key] = n * splits;
  return n * splits;
}

// Skinny-kernel configurations for C[m, n] (m <= 256) that run in ONE wave, fewest bytes per
// CTA first: (weight slice + activation rows of its K range) per CTA, plus its fp32 export.
std::vector<SkCfg> sk_candidates(int m, int n, int k, int act) {
  std::vector<SkCfg> out;
  if (m <= 0 || m > 256 || k % BK || (act && n % 32)) return out;
  const int np = ((m + 15) / 16) * 16;
  const int num_kb = k / BK;
  std::vector<std::pair<double, SkCfg>> scored;
  for (int shape = 0; shape < 3; ++shape) {
    // (rows per MMA, sub-tiles): (64, 1) doubles the CTAs of (128, 1) without splitting K
    const int mr = shape == 0 ? 64 : BM, mw = shape == 2 ? 2 : 1;
    if (mw * np > 512) continue;
    const int tiles = (n + mw * mr - 1) / (mw * mr);
    const int stage = mw * mr * BK * 2 + np * BK * 2;
    int prev = 0;
    for (int sp = 1; sp <= 8; ++sp) {
      const int kbs = (num_kb + sp - 1) / sp;
      const int s_eff = (num_kb + kbs - 1) / kbs;
      if (s_eff == prev) continue;
      prev = s_eff;
      // deepest ring that fits one CTA per SM, and the deepest that fits two
      for (int two = 0; two < 2; ++two) {
        const int budget = two ? DEC_SMEM_MAX / 2 - 2048 : DEC_SMEM_MAX;
        int st = (budget - 1024 - 8 * 20) / stage;
        if (st > 12) st = 12;
        if (st > kbs) st = kbs < 2 ? 2 : kbs;
        if (st < 2) continue;
        const int smem = sk_smem(np, mw, st, mr);
        if (smem > budget) continue;
        const int cap = sk_capacity(s_eff, smem);
        const int units = tiles * s_eff;
        if (units > cap) continue;  // one wave only
        SkCfg c{np, mw, s_eff, kbs, st, smem, tiles, mr};
        const double bytes = (double)kbs * stage + (s_eff > 1 ? 2.0 * np * mr * 4 * mw : 0.0);
        scored.push_back({bytes, c});
      }
    }
  }
  std::sort(scored.begin(), scored.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
  for (auto& s : scored) out.push_back(s.second);
  return out;
}

cudaError_t run_skinny(const SkCfg& d, const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc,
                       int m, int n, int k, cudaStream_t stream, int act = 0, const GemmRsEpilogue* rs = nullptr,
                       int blocked = 0, uint64_t* trace = nullptr) {
  if (m > 256 || k % BK || (act && n % 32) || ldc % 8) return cudaErrorInvalidValue;
  if (blocked && (n % BM || d.mrows != BM)) return cudaErrorInvalidValue;
  if (d.mrows != BM && (d.mrows != 64 || d.mw != 1)) return cudaErrorInvalidValue;
  CUtensorMap mx, mw;
  const bool wok = blocked ? make_map(&mw, w, n * (k / BK), BK, BK, BM) : make_map(&mw, w, n, k, ldw, d.mrows);
  if (!make_map(&mx, x, m, k, ldx, d.np) || !wok) return cudaErrorInvalidValue;
  SkParams p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.np = d.np;
  p.mrows = d.mrows;
  p.mw = d.mw;
  p.splits = d.splits;
  p.kb_per_split = d.kb_per_split;
  p.num_kb = k / BK;
  p.stages = d.stages;
  p.act = act;
  p.blocked = blocked;
  p.trace = trace;
  // D f32, A bf16 (weights), B bf16 (tokens), N = np, M = mrows
  p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(d.np >> 3) << 17) | ((uint32_t)(d.mrows >> 4) << 24);
  p.c = static_cast<__nv_bfloat16*>(c);
  p.ldc = ldc;
  if (rs) {
    if (act || rs->rows <= 0 || rs->world < 1 || rs->world > 8 || !rs->calls || !rs->ctas_done ||
        (int64_t)rs->rows * rs->world < m)
      return cudaErrorInvalidValue;
    for (int r = 0; r < rs->world; ++r)
      if (!rs->dst[r] || !rs->flag[r] || ((uintptr_t)rs->dst[r] & 15)) return cudaErrorInvalidValue;
    p.rs = *rs;
  } else if (!c || ((uintptr_t)c & 15)) {
    return cudaErrorInvalidValue;
  }
  static std::atomic<uint64_t> done{0};
  cudaError_t e = smem_opt_in(done, gemm_skinny_kernel, DEC_SMEM_MAX);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(d.tiles * d.splits, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = d.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = d.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, gemm_skinny_kernel, mw, mx, p);
}

}  // namespace

cudaError_t gemm_dec_explicit(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int m,
                              int n, int k, int bn, int splits, int a_stages, cudaStream_t stream) {
  for (const auto& d : dec_candidates(m, n, k))
    if (d.bn == bn && d.splits == splits && d.a_stages == a_stages)
      return run_dec(d, x, ldx, w, ldw, c, ldc, m, n, k, stream);
  return cudaErrorInvalidValue;
}

static GemmPlan dec_to_plan(const DecCfg& d, int k);

bool gemm_dec_plan(int m, int n, int k, int rank, GemmPlan* plan) {
  const auto cands = dec_candidates(m, n, k);
  if (rank < 0 || rank >= (int)cands.size()) return false;
  *plan = dec_to_plan(cands[rank], k);
  return true;
}

// Decode-kernel plans worth timing: the `each` cheapest by either model, plus the two narrowest
// single-split shapes that fill the GPU in one wave (no split-K reduction at all), deduplicated.
static std::vector<GemmPlan> dec_plans_for_tuning(int m, int n, int k, int each, int act) {
  std::vector<GemmPlan> out;
  {
    auto all = dec_candidates(m, n, k);
    std::vector<DecCfg> one;
    for (const auto& d : all)
      if (d.splits == 1 && d.tiles <= num_sms() && (!act || d.bn % 32 == 0)) one.push_back(d);
    std::sort(one.begin(), one.end(), [](const DecCfg& a, const DecCfg& b) {
      return a.bn != b.bn ? a.bn < b.bn : a.w_stages > b.w_stages;
    });
    int taken = 0;
    int last_bn = -1;
    for (const auto& d : one) {
      if (taken >= 2) break;
      if (d.bn == last_bn) continue;
      last_bn = d.bn;
      out.push_back(dec_to_plan(d, k));
      ++taken;
    }
  }
  for (int by_traffic = 0; by_traffic < 2; ++by_traffic) {
    int taken = 0;
    for (const auto& d : dec_candidates(m, n, k, by_traffic != 0)) {
      if (taken >= each) break;
      if (act && d.bn % 32) continue;
      bool dup = false;
      for (const auto& p : out)
        dup |= p.bn == d.bn && p.splits == d.splits && p.a_stages == d.a_stages && p.stages == d.w_stages;
      if (dup) continue;
      out.push_back(dec_to_plan(d, k));
      ++taken;
    }
  }
  return out;
}

// Skinny-kernel plans (dec = 2): mt = tokens per tile (MMA N), bn = weight rows per CTA.
// The `each` cheapest by bytes per CTA come first; the 64-row single-split shapes (more CTAs, no
// split-K reduction at all) are appended when the cheapest do not already include them.
static std::vector<GemmPlan> skinny_plans_for_tuning(int m, int n, int k, int each, int act) {
  std::vector<GemmPlan> out;
  const auto cands = sk_candidates(m, n, k, act);
  std::vector<SkCfg> pick;
  for (const auto& d : cands) {
    if ((int)pick.size() >= each) break;
    pick.push_back(d);
  }
  for (const auto& d : cands) {
    if (d.mrows != 64 || d.splits != 1) continue;
    bool dup = false;
    for (const auto& q : pick) dup |= q.mrows == d.mrows && q.splits == d.splits && q.stages == d.stages;
    if (!dup) pick.push_back(d);
  }
  for (const auto& d : pick) {
    GemmPlan pl{};
    pl.dec = 2;
    pl.mt = d.np;
    pl.bn = d.mw * d.mrows;
    pl.splits = d.splits;
    pl.kb_per_split = d.kb_per_split;
    pl.num_kb = k / BK;
    pl.stages = d.stages;
    pl.smem = d.smem;
    pl.tiles = d.tiles;
    pl.tiles_p = 1;
    pl.tiles_q = d.tiles;
    pl.grid = d.tiles * d.splits;
    out.push_back(pl);
  }
  return out;
}

bool gemm_skinny_plan(int m, int n, int k, int rank, int act, GemmPlan* plan) {
  const auto v = skinny_plans_for_tuning(m, n, k, rank + 1, act);
  if (rank < 0 || rank >= (int)v.size()) return false;
  *plan = v[rank];
  return true;
}

static SkCfg plan_to_skinny(const GemmPlan& pl) {
  // bn = weight rows per CTA: 64 (one 64-row MMA), 128 or 256 (one or two 128-row MMAs)
  const int mrows = pl.bn < BM ? 64 : BM;
  return SkCfg{pl.mt, pl.bn / mrows, pl.splits, pl.kb_per_split, pl.stages, pl.smem, pl.tiles, mrows};
}

cudaError_t gemm_skinny_run(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int m, int n,
                            int k, const GemmPlan& plan, int act, int blocked, cudaStream_t stream, uint64_t* trace) {
  if (plan.dec != 2) return cudaErrorInvalidValue;
  return run_skinny(plan_to_skinny(plan), x, ldx, w, ldw, c, ldc, m, n, k, stream, act, nullptr, blocked, trace);
}

// Pair-kernel plans (dec = 3): bn = weight rows per pair, tiles = pairs.
static std::vector<GemmPlan> pair_plans_for_tuning(int m, int n, int k, int each, int act) {
  std::vector<GemmPlan> out;
  for (const auto& d : pair_candidates(m, n, k, act)) {
    if ((int)out.size() >= each) break;
    GemmPlan pl{};
    pl.dec = 3;
    pl.mt = 2;
    pl.bn = d.bn;
    pl.splits = 1;
    pl.kb_per_split = k / BK;
    pl.num_kb = k / BK;
    pl.stages = d.stages;
    pl.smem = d.smem;
    pl.tiles = d.pairs;
    pl.tiles_p = 1;
    pl.tiles_q = d.pairs;
    pl.grid = 2 * d.pairs;
    out.push_back(pl);
  }
  return out;
}

bool gemm_pair_plan(int m, int n, int k, int rank, int act, GemmPlan* plan) {
  const auto v = pair_plans_for_tuning(m, n, k, rank + 1, act);
  if (rank < 0 || rank >= (int)v.size()) return false;
  *plan = v[rank];
  return true;
}

static GemmPlan dec_to_plan(const DecCfg& d, int k) {
  GemmPlan pl{};
  pl.dec = 1;
  pl.mt = d.mt;
  pl.bn = d.bn;
  pl.splits = d.splits;
  pl.kb_per_split = d.kb_per_split;
  pl.num_kb = k / BK;
  pl.stages = d.w_stages;
  pl.a_stages = d.a_stages;
  pl.smem = d.smem;
  pl.tiles = d.tiles;
  pl.tiles_p = 1;
  pl.tiles_q = d.tiles;
  pl.grid = d.tiles * d.splits;
  return pl;
}

GemmPlan gemm_plan(int m, int n, int k, int force_swap, int force_bn, int force_splits) {
  GemmPlan pl{};
  const int sms = num_sms();
  // Tokens always fill the 128-row MMA side: measured faster than the swapped form at
  // every batch size, because the weight tile then arrives in 256-row TMA boxes.
  pl.swap = force_swap >= 0 ? force_swap : 0;
  const int q_rows = pl.swap ? m : n;
  const int p_rows = pl.swap ? n : m;
  pl.num_kb = (k + BK - 1) / BK;
  int bn;
  if (force_bn > 0) {
    bn = force_bn;
  } else if (pl.swap) {
    bn = q_rows <= 32 ? 32 : q_rows <= 64 ? 64 : q_rows <= 128 ? 128 : 256;
  } else {
    // widest tile that still gives about one wave of tiles (decode-sized m: always 256)
    bn = 256;
    if ((p_rows + BM - 1) / BM > 2)
      while (bn > 128 && (int64_t)((p_rows + BM - 1) / BM) * ((q_rows + bn - 1) / bn) < (sms * 9) / 10) bn >>= 1;
  }
  pl.bn = bn;
  pl.mt = 1;
  pl.streamk = 0;
  if (force_splits < 0) {
    // stream-K over tiles of (128 * mt) x bn
    pl.mt = -force_splits > 1 ? 2 : 1;
    pl.streamk = 1;
    pl.tiles_p = (p_rows + BM * pl.mt - 1) / (BM * pl.mt);
    pl.tiles_q = (q_rows + bn - 1) / bn;
    pl.tiles = pl.tiles_p * pl.tiles_q;
    pl.splits = 1;
    pl.kb_per_split = pl.num_kb;
    const int64_t iters = (int64_t)pl.tiles * pl.num_kb;
    pl.grid = iters < sms ? (int)iters : sms;
    pl.ws_ld = bn;
    pl.ws_elems = (int64_t)pl.grid * 2 * pl.mt * BM * bn;
    pl.prefetch_w = (pl.swap ? pl.tiles_q : pl.tiles_p) <= 2;
    return pl;
  }
  pl.tiles_p = (p_rows + BM - 1) / BM;
  pl.tiles_q = (q_rows + bn - 1) / bn;
  const int tiles = pl.tiles_p * pl.tiles_q;
  int splits = 1;
  if (force_splits > 0) {
    splits = force_splits;
  } else {
    // Rounds x k-blocks per CTA plus a fixed per-CTA cost; split-K runs as clusters whose
    // concurrency is what the driver reports for the cluster shape.
    auto cost = [&](int sp) {
      const int kbs = (pl.num_kb + sp - 1) / sp;
      const int units = tiles * sp;
      const int cap = sp > 1 ? cluster_capacity(bn, sp) : sms;
      const int waves = (units + cap - 1) / (cap > 0 ? cap : 1);
      return (double)waves * (kbs + (sp > 1 ? 6 : 2));
    };
    double best = cost(1);
    for (int sp = 2; sp <= 8; ++sp) {
      if (pl.num_kb / sp < 2) break;
      const double c = cost(sp);
      if (c < best * 0.97) {
        best = c;
        splits = sp;
      }
    }
  }
  if (splits > 8) splits = 8;
  pl.kb_per_split = (pl.num_kb + splits - 1) / splits;
  pl.splits = (pl.num_kb + pl.kb_per_split - 1) / pl.kb_per_split;
  const int units = tiles * pl.splits;
  pl.grid = units < sms ? units : sms;
  pl.ws_ld = 0;
  pl.ws_elems = 0;  // split-K reduces through distributed shared memory: no scratch
  pl.tiles = tiles;
  pl.prefetch_w = (pl.swap ? pl.tiles_q : pl.tiles_p) <= 2;
  return pl;
}

bool sample_plan_ok(const GemmPlan& pl) { return !pl.dec && (pl.streamk || pl.splits <= 1); }

cudaError_t gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int m, int n, int k,
                      const GemmPlan& pl, float* ws, int* counters, cudaStream_t stream, int act,
                      const GemmSampleEpilogue* se) {
  if (m == 0 || n == 0) return cudaSuccess;
  if (act && (pl.swap || n % 32 || pl.bn % 32)) return cudaErrorInvalidValue;
  if (k % 8 || ldx % 8 || ldw % 8) return cudaErrorInvalidValue;
  if (((uintptr_t)x & 15) || ((uintptr_t)w & 15)) return cudaErrorMisalignedAddress;
  if (se) {  // the sampling epilogue lives in the persistent kernel (one K range per tile, or stream-K)
    if (act || !sample_plan_ok(pl) || !se->keys || !se->temps || !se->seed_step) return cudaErrorInvalidValue;
  } else if (!pl.swap && (ldc % 8 || ((uintptr_t)c & 15))) {
    return cudaErrorInvalidValue;
  }
  if (pl.dec == 2) {
    if (m > pl.mt || k % BK) return cudaErrorInvalidValue;
    return run_skinny(plan_to_skinny(pl), x, ldx, w, ldw, c, ldc, m, n, k, stream, act);
  }
  if (pl.dec == 3) return run_pair(PairCfg{pl.bn, pl.stages, pl.smem, pl.tiles}, x, ldx, w, ldw, c, ldc, m, n, k, stream, act);
  if (pl.dec) {
    if (m > pl.mt * BM || k % BK) return cudaErrorInvalidValue;
    DecCfg d{pl.mt, pl.bn, pl.splits, pl.kb_per_split, pl.stages, pl.a_stages, pl.smem, pl.tiles, 0.0};
    return run_dec(d, x, ldx, w, ldw, c, ldc, m, n, k, stream, act);
  }
  const void* pbase = pl.swap ? w : x;
  const void* qbase = pl.swap ? x : w;
  const int64_t pld = pl.swap ? ldw : ldx, qld = pl.swap ? ldx : ldw;
  const int p_rows = pl.swap ? n : m, q_rows = pl.swap ? m : n;
  CUtensorMap mp, mq;
  if (!make_map(&mp, pbase, p_rows, k, pld, BM) || !make_map(&mq, qbase, q_rows, k, qld, pl.bn))
    return cudaErrorInvalidValue;
  Params prm;
  prm.p_rows = p_rows;
  prm.q_rows = q_rows;
  prm.k = k;
  prm.tiles_p = pl.tiles_p;
  prm.tiles_q = pl.tiles_q;
  prm.splits = pl.splits;
  prm.kb_per_split = pl.kb_per_split;
  prm.num_kb = pl.num_kb;
  prm.swap = pl.swap;
  prm.prefetch_w = pl.prefetch_w;
  prm.group = 16;
  prm.c = static_cast<__nv_bfloat16*>(c);
  prm.ldc = ldc;
  prm.ws = ws;
  prm.ws_ld = pl.ws_ld;
  prm.counters = counters;
  prm.streamk = pl.streamk;
  prm.act = act;
  prm.keys = se ? se->keys : nullptr;
  prm.temps = se ? se->temps : nullptr;
  prm.seed_step = se ? se->seed_step : nullptr;
  prm.col_offset = se ? se->col_offset : 0;
  prm.sk_iters = (int64_t)pl.tiles * pl.num_kb;
  cudaError_t e;
  if (pl.streamk) {
    if (!ws || !counters) return cudaErrorInvalidValue;
    if (pl.mt == 2) {
      switch (pl.bn) {
        case 128: return run<128, 2>(mp, mq, prm, pl.grid, stream);
        case 256: return run<256, 2>(mp, mq, prm, pl.grid, stream);
        default: return cudaErrorInvalidValue;
      }
    }
    switch (pl.bn) {
      case 64: return run<64>(mp, mq, prm, pl.grid, stream);
      case 128: return run<128>(mp, mq, prm, pl.grid, stream);
      case 256: return run<256>(mp, mq, prm, pl.grid, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  if (pl.splits > 1) {
    switch (pl.bn) {
      case 32: return run_cluster<32>(mp, mq, prm, stream);
      case 64: return run_cluster<64>(mp, mq, prm, stream);
      case 128: return run_cluster<128>(mp, mq, prm, stream);
      case 256: return run_cluster<256>(mp, mq, prm, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (pl.bn) {
    case 32: e = run<32>(mp, mq, prm, pl.grid, stream); break;
    case 64: e = run<64>(mp, mq, prm, pl.grid, stream); break;
    case 128: e = run<128>(mp, mq, prm, pl.grid, stream); break;
    case 256: e = run<256>(mp, mq, prm, pl.grid, stream); break;
    default: return cudaErrorInvalidValue;
  }
  return e;
}

// ---------------------------------------------------------------- autotuning
// Key: (m bucket, n, k).  m <= 256 is keyed exactly (decode batch buckets); larger m
// by multiples of 512.
namespace {
// Reads a buffer larger than L2 so that the next launch finds its operands in HBM and L2
// holds only clean lines (a write would leave dirty lines whose write-back the timed
// launch would pay for).
__global__ void l2_evict_kernel(const uint4* __restrict__ p, size_t n, int* __restrict__ sink) {
  uint32_t acc = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const uint4 v = p[i];
    acc ^= v.x ^ v.y ^ v.z ^ v.w;
  }
  if (acc == 0x9E3779B9u) *sink = (int)acc;  // keeps the loads; the value is irrelevant
}

std::map<std::tuple<int, int, int>, GemmPlan>& tune_cache() {
  static std::map<std::tuple<int, int, int>, GemmPlan> c;
  return c;
}
std::mutex& tune_mutex() {
  static std::mutex mu;
  return mu;
}
int m_bucket(int m) { return m <= 256 ? m : ((m + 511) / 512) * 512; }

// Deterministic mode: plans come from the shape alone (no timing), so every process computes a
// shape with the same kernel and the same split-K order (bit-identical results across the
// processes of a P/D pair or a TP group).  Default from the environment (NVB_DETERMINISTIC=1).
std::atomic<int>& deterministic_flag() {
  static std::atomic<int> f{[] {
    const char* e = getenv("NVB_DETERMINISTIC");
    return e && e[0] && e[0] != '0' ? 1 : 0;
  }()};
  return f;
}
}  // namespace

void gemm_set_deterministic(int on) { deterministic_flag().store(on ? 1 : 0); }
int gemm_deterministic() { return deterministic_flag().load(); }

cudaError_t gemm_bf16_tuned(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int m, int n,
                            int k, float* ws, int64_t ws_elems, int* counters, int64_t num_counters,
                            cudaStream_t stream, GemmPlan* chosen, int act) {
  if (m == 0 || n == 0) return cudaSuccess;
  if (gemm_deterministic()) {  // the shape alone decides, whatever was tuned before
    const GemmPlan pl = gemm_plan(m, n, k, act ? 0 : -1, 0, 0);
    if (chosen) *chosen = pl;
    return gemm_bf16(x, ldx, w, ldw, c, ldc, m, n, k, pl, ws, counters, stream, act);
  }
  const auto key = std::make_tuple(m_bucket(m), act ? -n : n, k);
  {
    std::lock_guard<std::mutex> g(tune_mutex());
    auto it = tune_cache().find(key);
    if (it != tune_cache().end()) {
      if (chosen) *chosen = it->second;
      return gemm_bf16(x, ldx, w, ldw, c, ldc, m, n, k, it->second, ws, counters, stream, act);
    }
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(stream, &cap);
  GemmPlan best = gemm_plan(m, n, k, act ? 0 : -1, 0, 0);
  if (cap != cudaStreamCaptureStatusNone || gemm_deterministic()) {  // no timing: capture or deterministic
    if (chosen) *chosen = best;
    return gemm_bf16(x, ldx, w, ldw, c, ldc, m, n, k, best, ws, counters, stream, act);
  }
  std::vector<GemmPlan> cands;
  cands.push_back(best);
  for (int bn : {256, 128})
    for (int sp : {1, 2, 3, 4, 6, 8}) cands.push_back(gemm_plan(m, n, k, 0, bn, sp));
  if (m <= 256 && !act) {
    const int bq = m <= 32 ? 32 : m <= 64 ? 64 : m <= 128 ? 128 : 256;
    for (int sp : {1, 2, 3, 4}) cands.push_back(gemm_plan(m, n, k, 1, bq, sp));
  }
  if (m <= 2 * BM && k % BK == 0) {
    for (const auto& d : dec_plans_for_tuning(m, n, k, 6, act)) cands.push_back(d);
    for (const auto& d : skinny_plans_for_tuning(m, n, k, 6, act)) cands.push_back(d);
    for (const auto& d : pair_plans_for_tuning(m, n, k, 6, act)) cands.push_back(d);
  }
  if (ws && counters) {
    for (int bn : {256, 128}) {
      cands.push_back(gemm_plan(m, n, k, 0, bn, -1));
      if (m > BM) cands.push_back(gemm_plan(m, n, k, 0, bn, -2));
    }
  }
  // Each candidate is timed on a cold L2 (the weights of a real forward pass are not
  // resident when their layer runs): a 256 MiB read precedes every timed launch.
  const size_t flush_bytes = (size_t)256 << 20;
  void* flush = nullptr;
  if (cudaMalloc(&flush, flush_bytes) != cudaSuccess) {
    cudaGetLastError();
    flush = nullptr;
  }
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  float best_ms = 1e30f;
  for (const auto& pl : cands) {
    if (pl.splits > 1 && pl.splits > 8) continue;
    if (pl.streamk && (pl.ws_elems > ws_elems || 4 * (int64_t)pl.tiles > num_counters)) continue;
    if (gemm_bf16(x, ldx, w, ldw, c, ldc, m, n, k, pl, ws, counters, stream, act) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    float total = 0.f;
    bool good = true;
    for (int r = 0; r < 3 && good; ++r) {
      if (flush)
        l2_evict_kernel<<<num_sms() * 4, 256, 0, stream>>>(static_cast<const uint4*>(flush), flush_bytes / 16 - 16,
                                                          static_cast<int*>(flush) + (flush_bytes / 4 - 1));
      cudaEventRecord(e0, stream);
      good = gemm_bf16(x, ldx, w, ldw, c, ldc, m, n, k, pl, ws, counters, stream, act) == cudaSuccess;
      cudaEventRecord(e1, stream);
      cudaEventSynchronize(e1);
      float ms = 0.f;
      cudaEventElapsedTime(&ms, e0, e1);
      total += ms;
    }
    if (good && total < best_ms) {
      best_ms = total;
      best = pl;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (flush) cudaFree(flush);
  {
    std::lock_guard<std::mutex> g(tune_mutex());
    tune_cache()[key] = best;
  }
  if (chosen) *chosen = best;
  return gemm_bf16(x, ldx, w, ldw, c, ldc, m, n, k, best, ws, counters, stream, act);
}

cudaError_t gemm_bf16_sample(const void* x, int64_t ldx, const void* w, int64_t ldw, int m, int n, int k,
                             const GemmSampleEpilogue& se, float* ws, int64_t ws_elems, int* counters,
                             int64_t num_counters, bool tune, cudaStream_t stream, GemmPlan* chosen) {
  if (m == 0 || n == 0) return cudaSuccess;
  static std::map<std::tuple<int, int, int>, GemmPlan> cache;  // guarded by tune_mutex()
  const auto key = std::make_tuple(m_bucket(m), n, k);
  auto fits = [&](const GemmPlan& pl) {
    return sample_plan_ok(pl) && (!pl.streamk || (ws && counters && pl.ws_elems <= ws_elems &&
                                                  4 * (int64_t)pl.tiles <= num_counters));
  };
  // the plain GEMM's heuristic plan when the persistent kernel runs it (deterministic mode then
  // rounds every logit as the logits path does), else the heuristic orientation with one K range
  GemmPlan best = gemm_plan(m, n, k, -1, 0, 0);
  if (!sample_plan_ok(best)) best = gemm_plan(m, n, k, -1, 0, 1);
  {
    std::lock_guard<std::mutex> g(tune_mutex());
    auto it = cache.find(key);
    if (it != cache.end()) {
      if (chosen) *chosen = it->second;
      return gemm_bf16(x, ldx, w, ldw, nullptr, 0, m, n, k, it->second, ws, counters, stream, 0, &se);
    }
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(stream, &cap);
  if (tune && cap == cudaStreamCaptureStatusNone && !gemm_deterministic()) {
    // time the persistent-kernel candidates with the sampling epilogue itself (its cost depends on
    // the orientation), each after a 256 MiB read, then clear the keys they left behind
    std::vector<GemmPlan> cands{best};
    for (int bn : {256, 128}) cands.push_back(gemm_plan(m, n, k, 0, bn, 1));
    if (m <= 256) cands.push_back(gemm_plan(m, n, k, 1, m <= 32 ? 32 : m <= 64 ? 64 : m <= 128 ? 128 : 256, 1));
    for (int bn : {256, 128}) {
      cands.push_back(gemm_plan(m, n, k, 0, bn, -1));
      if (m > BM) cands.push_back(gemm_plan(m, n, k, 0, bn, -2));
    }
    const size_t flush_bytes = (size_t)256 << 20;
    void* flush = nullptr;
    if (cudaMalloc(&flush, flush_bytes) != cudaSuccess) {
      cudaGetLastError();
      flush = nullptr;
    }
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    float best_ms = 1e30f;
    for (const auto& pl : cands) {
      if (!fits(pl)) continue;
      if (gemm_bf16(x, ldx, w, ldw, nullptr, 0, m, n, k, pl, ws, counters, stream, 0, &se) != cudaSuccess) {
        cudaGetLastError();
        continue;
      }
      float total = 0.f;
      bool good = true;
      for (int r = 0; r < 3 && good; ++r) {
        if (flush)
          l2_evict_kernel<<<num_sms() * 4, 256, 0, stream>>>(static_cast<const uint4*>(flush), flush_bytes / 16 - 16,
                                                            static_cast<int*>(flush) + (flush_bytes / 4 - 1));
        cudaEventRecord(e0, stream);
        good = gemm_bf16(x, ldx, w, ldw, nullptr, 0, m, n, k, pl, ws, counters, stream, 0, &se) == cudaSuccess;
        cudaEventRecord(e1, stream);
        cudaEventSynchronize(e1);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        total += ms;
      }
      if (good && total < best_ms) {
        best_ms = total;
        best = pl;
      }
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (flush) cudaFree(flush);
    cudaMemsetAsync(se.keys, 0, sizeof(unsigned long long) * (size_t)m, stream);
    std::lock_guard<std::mutex> g(tune_mutex());
    cache[key] = best;
  } else if (!fits(best)) {
    best = gemm_plan(m, n, k, 0, 128, 1);
  }
  if (chosen) *chosen = best;
  return gemm_bf16(x, ldx, w, ldw, nullptr, 0, m, n, k, best, ws, counters, stream, 0, &se);
}

cudaError_t gemm_bf16_rs(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t ldc, int m, int n, int k,
                         const GemmRsEpilogue& rs, void* tune_c, int64_t tune_ldc, cudaStream_t stream,
                         GemmPlan* chosen) {
  if (m == 0 || n == 0) return cudaSuccess;
  if (m > 2 * BM || k % BK || k % 8 || ldx % 8 || ldw % 8) return cudaErrorNotSupported;
  if (((uintptr_t)x & 15) || ((uintptr_t)w & 15)) return cudaErrorMisalignedAddress;
  static std::map<std::tuple<int, int, int>, GemmPlan> cache;  // guarded by tune_mutex()
  const auto key = std::make_tuple(m, n, k);
  GemmPlan best{};
  bool have = false;
  if (!gemm_deterministic()) {
    std::lock_guard<std::mutex> g(tune_mutex());
    auto it = cache.find(key);
    if (it != cache.end()) {
      best = it->second;
      have = true;
    }
  }
  if (!have) {
    std::vector<GemmPlan> cands = dec_plans_for_tuning(m, n, k, 6, 0);
    for (const auto& d : skinny_plans_for_tuning(m, n, k, 6, 0)) cands.push_back(d);
    if (cands.empty()) return cudaErrorNotSupported;
    best = cands[0];
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(stream, &cap);
    if (cap == cudaStreamCaptureStatusNone && tune_c && cands.size() > 1 && !gemm_deterministic()) {
      // time the candidates with a plain local output (the reduce-scatter stores and flags
      // must only happen once per reduction), each after a 256 MiB read (cold L2)
      const size_t flush_bytes = (size_t)256 << 20;
      void* flush = nullptr;
      if (cudaMalloc(&flush, flush_bytes) != cudaSuccess) {
        cudaGetLastError();
        flush = nullptr;
      }
      cudaEvent_t e0, e1;
      cudaEventCreate(&e0);
      cudaEventCreate(&e1);
      float best_ms = 1e30f;
      for (const auto& pl : cands) {
        if (gemm_bf16(x, ldx, w, ldw, tune_c, tune_ldc, m, n, k, pl, nullptr, nullptr, stream, 0) != cudaSuccess) {
          cudaGetLastError();
          continue;
        }
        float total = 0.f;
        bool good = true;
        for (int r = 0; r < 3 && good; ++r) {
          if (flush)
            l2_evict_kernel<<<num_sms() * 4, 256, 0, stream>>>(static_cast<const uint4*>(flush), flush_bytes / 16 - 16,
                                                              static_cast<int*>(flush) + (flush_bytes / 4 - 1));
          cudaEventRecord(e0, stream);
          good = gemm_bf16(x, ldx, w, ldw, tune_c, tune_ldc, m, n, k, pl, nullptr, nullptr, stream, 0) == cudaSuccess;
          cudaEventRecord(e1, stream);
          cudaEventSynchronize(e1);
          float ms = 0.f;
          cudaEventElapsedTime(&ms, e0, e1);
          total += ms;
        }
        if (good && total < best_ms) {
          best_ms = total;
          best = pl;
        }
      }
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
      if (flush) cudaFree(flush);
      std::lock_guard<std::mutex> g(tune_mutex());
      cache[key] = best;
    }
  }
  if (chosen) *chosen = best;
  if (best.dec == 2) return run_skinny(plan_to_skinny(best), x, ldx, w, ldw, nullptr, ldc, m, n, k, stream, 0, &rs);
  DecCfg dc{best.mt, best.bn, best.splits, best.kb_per_split, best.stages, best.a_stages, best.smem, best.tiles, 0.0};
  return run_dec(dc, x, ldx, w, ldw, nullptr, ldc, m, n, k, stream, 0, &rs);
}

int gemm_error_code(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_gemm_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace nvb
