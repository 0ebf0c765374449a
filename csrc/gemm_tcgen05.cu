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
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > WAIT_BUDGET_NS) {
      atomicCAS(&g_gemm_error, 0, code);
      *abort_flag = 1;
      return false;
    }
  }
}

// Drain wait used on the error path: short budget, never sets flags.
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try(bar, parity)) {
    if (globaltimer() - t0 > WAIT_BUDGET_NS) return;
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
};

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

// Store 32 accumulator columns [qc, qc + 32) of accumulator row pi as bf16.
__device__ __forceinline__ void store_chunk(const Params& p, int pi, int qc, const float* f) {
  if (pi >= p.p_rows) return;
  if (!p.swap) {
    __nv_bfloat16* dst = p.c + (int64_t)pi * p.ldc + qc;
    const int valid = p.q_rows - qc;
    if (valid >= 32) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) *reinterpret_cast<uint4*>(dst + j) = f32_to_bf16x8(f + j);
    } else {
      for (int j = 0; j < valid; ++j) dst[j] = __float2bfloat16(f[j]);
    }
  } else {
    // C[j, pi]: the 32 lanes of a warp hold consecutive pi, so each store is coalesced
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (qc + j < p.q_rows) p.c[(int64_t)(qc + j) * p.ldc + pi] = __float2bfloat16(f[j]);
  }
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_p, const __grid_constant__ CUtensorMap map_q, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int P_BYTES = BM * BK * 2;
  constexpr int Q_BYTES = BN * BK * 2;
  constexpr int STAGE_BYTES = P_BYTES + Q_BYTES;
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
  constexpr uint32_t TMEM_COLS = 2 * BN;

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

  const int total_units = p.tiles_p * p.tiles_q * p.splits;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_p)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_q)) : "memory");
      uint32_t it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        int tp, tq, sp;
        unit_coords(p, u, tp, tq, sp);
        const int kb0 = sp * p.kb_per_split, nkb = min(p.num_kb, kb0 + p.kb_per_split) - kb0;
        const int rot = (tp + tq) % nkb;
        const CUtensorMap* wmap = p.swap ? &map_p : &map_q;
        const int wrow = p.swap ? tp * BM : tq * BN;
        if (p.prefetch_w)
          for (int i = 0; i < min(nkb, PF_DIST); ++i) tma_prefetch_2d(wmap, (kb0 + (i + rot) % nkb) * BK, wrow);
        for (int i = 0; i < nkb; ++i, ++it) {
          const int kb = kb0 + (i + rot) % nkb;
          const int s = it % STAGES;
          const uint32_t round = it / STAGES;
          if (p.prefetch_w && i + PF_DIST < nkb) tma_prefetch_2d(wmap, (kb0 + (i + PF_DIST + rot) % nkb) * BK, wrow);
          if (!mbar_wait(empty(s), (round & 1) ^ 1, abort_flag, 1)) {
            ok = false;
            break;
          }
          const uint32_t st = smem_u32(smem + s * STAGE_BYTES);
          mbar_arrive_expect_tx(full(s), STAGE_BYTES);
          tma_load_2d(st, &map_p, full(s), kb * BK, tp * BM);
          tma_load_2d(st + P_BYTES, &map_q, full(s), kb * BK, tq * BN);
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
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++tile_it) {
        int tp, tq, sp;
        unit_coords(p, u, tp, tq, sp);
        const int kb0 = sp * p.kb_per_split, nkb = min(p.num_kb, kb0 + p.kb_per_split) - kb0;
        const int acc = tile_it & 1;
        const uint32_t use = tile_it >> 1;
        if (!mbar_wait(tempty(acc), (use & 1) ^ 1, abort_flag, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int i = 0; i < nkb; ++i, ++it) {
          const int s = it % STAGES;
          const uint32_t round = it / STAGES;
          if (!mbar_wait(full(s), round & 1, abort_flag, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + s * STAGE_BYTES);
          const uint64_t pd = sdesc(st), qd = sdesc(st + P_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // advance 16 elements (32 bytes) along K inside the swizzle atom: +2 in the
            // 16-byte-unit start address field
            tc_mma(d_tmem, pd + 2 * k, qd + 2 * k, IDESC, (i > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(empty(s));
        }
        if (!ok) break;
        tc_commit(tfull(acc));
      }
      // Make sure every issued MMA has finished before TMEM is released.
      tc_commit(final_bar);
      mbar_drain(final_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int q4 = warp & 3;            // TMEM lane quarter this warp may access
    const int row = q4 * 32 + lane;     // accumulator row (P index within the tile)
    uint32_t tile_it = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++tile_it) {
      int tp, tq, sp;
      unit_coords(p, u, tp, tq, sp);
      const int acc = tile_it & 1;
      const uint32_t use = tile_it >> 1;
      if (!mbar_wait(tfull(acc), use & 1, abort_flag, 4)) break;
      tc_fence_after();
      const int pi = tp * BM + row;
      const int q0 = tq * BN;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(q4 * 32) << 16) + acc * BN + c0, r);
        float f[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
        store_chunk(p, pi, q0 + c0, f);
      }
      tc_fence_before();
      if (lane == 0) mbar_arrive(tempty(acc));
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
        tc_fence_after();
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
  // Each item is 4 consecutive columns of one row; all peers' float4 loads for an item
  // are issued before they are summed.
  for (int idx = threadIdx.x; idx < total; idx += NUM_THREADS) {
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

bool make_map(CUtensorMap* m, const void* base, int rows, int k, int64_t ld_elems, int box_rows) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld_elems * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN>
constexpr int stages_for() {
  return (200 * 1024) / (BM * BK * 2 + BN * BK * 2) > 8 ? 8 : (200 * 1024) / (BM * BK * 2 + BN * BK * 2);
}

template <int BN>
cudaError_t run_cluster(const CUtensorMap& mp, const CUtensorMap& mq, const Params& prm, cudaStream_t stream) {
  constexpr int STAGES = stages_for<BN>();
  constexpr int SMEM = STAGES * (BM * BK * 2 + BN * BK * 2) + 1024 + 256;
  auto kern = gemm_cluster_kernel<BN, STAGES>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(prm.tiles_p * prm.tiles_q * prm.splits, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = prm.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, mp, mq, prm);
}

template <int BN>
cudaError_t run(const CUtensorMap& mp, const CUtensorMap& mq, const Params& prm, int grid, cudaStream_t stream) {
  constexpr int STAGES = stages_for<BN>();
  constexpr int SMEM = STAGES * (BM * BK * 2 + BN * BK * 2) + 1024 + 256;
  auto kern = gemm_kernel<BN, STAGES>;
  static bool configured = false;  // per template instance; the attribute is process-wide
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  kern<<<grid, NUM_THREADS, SMEM, stream>>>(mp, mq, prm);
  return cudaGetLastError();
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int BN>
int max_active_clusters(int splits) {
  // CTAs of `splits`-wide clusters that can be resident at once (cached per size).
  static int cache[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
  if (splits < 2 || splits > 8) return 0;
  if (cache[splits]) return cache[splits];
  constexpr int STAGES = stages_for<BN>();
  constexpr int SMEM = STAGES * (BM * BK * 2 + BN * BK * 2) + 1024 + 256;
  auto kern = gemm_cluster_kernel<BN, STAGES>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits * 64, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = num_sms() / splits;
  }
  cache[splits] = n * splits;
  return cache[splits];
}

int cluster_capacity(int bn, int splits) {
  switch (bn) {
    case 32: return max_active_clusters<32>(splits);
    case 64: return max_active_clusters<64>(splits);
    case 128: return max_active_clusters<128>(splits);
    default: return max_active_clusters<256>(splits);
  }
}

}  // namespace

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

cudaError_t gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int m, int n, int k,
                      const GemmPlan& pl, float* ws, int* counters, cudaStream_t stream) {
  if (m == 0 || n == 0) return cudaSuccess;
  if (k % 8 || ldx % 8 || ldw % 8) return cudaErrorInvalidValue;
  if (((uintptr_t)x & 15) || ((uintptr_t)w & 15)) return cudaErrorMisalignedAddress;
  if (!pl.swap && (ldc % 8 || ((uintptr_t)c & 15))) return cudaErrorInvalidValue;
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
  (void)ws;
  (void)counters;
  cudaError_t e;
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
std::map<std::tuple<int, int, int>, GemmPlan>& tune_cache() {
  static std::map<std::tuple<int, int, int>, GemmPlan> c;
  return c;
}
std::mutex& tune_mutex() {
  static std::mutex mu;
  return mu;
}
int m_bucket(int m) { return m <= 256 ? m : ((m + 511) / 512) * 512; }
}  // namespace

cudaError_t gemm_bf16_tuned(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int m, int n,
                            int k, cudaStream_t stream, GemmPlan* chosen) {
  if (m == 0 || n == 0) return cudaSuccess;
  const auto key = std::make_tuple(m_bucket(m), n, k);
  {
    std::lock_guard<std::mutex> g(tune_mutex());
    auto it = tune_cache().find(key);
    if (it != tune_cache().end()) {
      if (chosen) *chosen = it->second;
      return gemm_bf16(x, ldx, w, ldw, c, ldc, m, n, k, it->second, nullptr, nullptr, stream);
    }
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(stream, &cap);
  GemmPlan best = gemm_plan(m, n, k, -1, 0, 0);
  if (cap != cudaStreamCaptureStatusNone) {  // cannot time inside a capture
    if (chosen) *chosen = best;
    return gemm_bf16(x, ldx, w, ldw, c, ldc, m, n, k, best, nullptr, nullptr, stream);
  }
  std::vector<GemmPlan> cands;
  cands.push_back(best);
  for (int bn : {256, 128})
    for (int sp : {1, 2, 3, 4, 6, 8}) cands.push_back(gemm_plan(m, n, k, 0, bn, sp));
  if (m <= 256) {
    const int bq = m <= 32 ? 32 : m <= 64 ? 64 : m <= 128 ? 128 : 256;
    for (int sp : {1, 2, 3, 4}) cands.push_back(gemm_plan(m, n, k, 1, bq, sp));
  }
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  float best_ms = 1e30f;
  for (const auto& pl : cands) {
    if (pl.splits > 1 && pl.splits > 8) continue;
    if (gemm_bf16(x, ldx, w, ldw, c, ldc, m, n, k, pl, nullptr, nullptr, stream) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    cudaEventRecord(e0, stream);
    for (int r = 0; r < 3; ++r) gemm_bf16(x, ldx, w, ldw, c, ldc, m, n, k, pl, nullptr, nullptr, stream);
    cudaEventRecord(e1, stream);
    cudaEventSynchronize(e1);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    if (ms < best_ms) {
      best_ms = ms;
      best = pl;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  {
    std::lock_guard<std::mutex> g(tune_mutex());
    tune_cache()[key] = best;
  }
  if (chosen) *chosen = best;
  return gemm_bf16(x, ldx, w, ldw, c, ldc, m, n, k, best, nullptr, nullptr, stream);
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
