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
// t overlaps the main loop of tile t+1.  With splits > 1 each unit writes an fp32
// partial tile to scratch and gemm_splitk_reduce sums the partials.
//
// Every mbarrier wait is bounded by a wall-clock budget; on expiry the kernel records
// an error code in a device word (read by gemm_error_code()), stops issuing work,
// drains its own copies and MMAs with bounded waits, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemm.h"

namespace nvb {

__device__ int g_gemm_error = 0;

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int NUM_THREADS = 192;
constexpr uint64_t WAIT_BUDGET_NS = 2000000000ull;  // 2 s

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
  int group;                 // tile rasterisation group along P
  __nv_bfloat16* c;
  int64_t ldc;
  float* ws;                 // split-K partials [splits][p_rows][q_rows_pad]
  int64_t ws_ld;
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
        const int kb0 = sp * p.kb_per_split, kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t round = it / STAGES;
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
        const int kb0 = sp * p.kb_per_split, kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        const int acc = tile_it & 1;
        const uint32_t use = tile_it >> 1;
        if (!mbar_wait(tempty(acc), (use & 1) ^ 1, abort_flag, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
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
            tc_mma(d_tmem, pd + 2 * k, qd + 2 * k, IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
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
        if (pi >= p.p_rows) continue;
        if (p.splits > 1) {
          float* dst = p.ws + ((int64_t)sp * p.p_rows + pi) * p.ws_ld + q0 + c0;
          if (q0 + c0 + 32 <= p.ws_ld) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(dst + j) = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                                __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
          }
        } else if (!p.swap) {
          __nv_bfloat16* dst = p.c + (int64_t)pi * p.ldc + q0 + c0;
          const int valid = p.q_rows - (q0 + c0);
          if (valid >= 32) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              float f[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[j + e]);
              *reinterpret_cast<uint4*>(dst + j) = f32_to_bf16x8(f);
            }
          } else {
            for (int j = 0; j < valid; ++j) dst[j] = __float2bfloat16(__uint_as_float(r[j]));
          }
        } else {
          // C[j, pi] for the token columns j of this chunk
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int qj = q0 + c0 + j;
            if (qj < p.q_rows) p.c[(int64_t)qj * p.ldc + pi] = __float2bfloat16(__uint_as_float(r[j]));
          }
        }
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

// Sum split-K partials [splits][p_rows][ws_ld] -> bf16 C (normal or swapped orientation).
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int64_t ws_ld, int splits, int p_rows, int q_rows,
                                     int swap, __nv_bfloat16* __restrict__ c, int64_t ldc) {
  const int64_t total = (int64_t)p_rows * q_rows;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    int i, j;
    if (swap) {  // walk output-contiguous: j = token (slow), i = feature (fast)
      j = (int)(idx / p_rows);
      i = (int)(idx - (int64_t)j * p_rows);
    } else {
      i = (int)(idx / q_rows);
      j = (int)(idx - (int64_t)i * q_rows);
    }
    float s = 0.f;
    for (int sp = 0; sp < splits; ++sp) s += ws[((int64_t)sp * p_rows + i) * ws_ld + j];
    if (swap)
      c[(int64_t)j * ldc + i] = __float2bfloat16(s);
    else
      c[(int64_t)i * ldc + j] = __float2bfloat16(s);
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

}  // namespace

GemmPlan gemm_plan(int m, int n, int k, int force_swap, int force_bn, int force_splits) {
  GemmPlan pl{};
  const int sms = num_sms();
  pl.swap = force_swap >= 0 ? force_swap : (m <= 256 ? 1 : 0);
  const int q_rows = pl.swap ? m : n;
  const int p_rows = pl.swap ? n : m;
  int bn;
  if (force_bn > 0) {
    bn = force_bn;
  } else if (pl.swap) {
    bn = q_rows <= 32 ? 32 : q_rows <= 64 ? 64 : q_rows <= 128 ? 128 : 256;
  } else {
    bn = 256;
  }
  pl.bn = bn;
  pl.tiles_p = (p_rows + BM - 1) / BM;
  pl.tiles_q = (q_rows + bn - 1) / bn;
  pl.num_kb = (k + BK - 1) / BK;
  const int tiles = pl.tiles_p * pl.tiles_q;
  int splits = 1;
  if (force_splits > 0) {
    splits = force_splits;
  } else if (tiles < sms) {
    splits = (sms + tiles - 1) / tiles;
    const int max_by_k = pl.num_kb / 4 > 0 ? pl.num_kb / 4 : 1;
    if (splits > max_by_k) splits = max_by_k;
    if (splits > 16) splits = 16;
  }
  pl.kb_per_split = (pl.num_kb + splits - 1) / splits;
  pl.splits = (pl.num_kb + pl.kb_per_split - 1) / pl.kb_per_split;
  const int units = tiles * pl.splits;
  pl.grid = units < sms ? units : sms;
  pl.ws_ld = (int64_t)pl.tiles_q * bn;
  pl.ws_elems = pl.splits > 1 ? (int64_t)pl.splits * p_rows * pl.ws_ld : 0;
  return pl;
}

cudaError_t gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int m, int n, int k,
                      const GemmPlan& pl, float* ws, cudaStream_t stream) {
  if (m == 0 || n == 0) return cudaSuccess;
  if (k % 8 || ldx % 8 || ldw % 8) return cudaErrorInvalidValue;
  if (((uintptr_t)x & 15) || ((uintptr_t)w & 15)) return cudaErrorMisalignedAddress;
  if (pl.splits > 1 && !ws) return cudaErrorInvalidValue;
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
  prm.group = 16;
  prm.c = static_cast<__nv_bfloat16*>(c);
  prm.ldc = ldc;
  prm.ws = ws;
  prm.ws_ld = pl.ws_ld;
  cudaError_t e;
  switch (pl.bn) {
    case 32: e = run<32>(mp, mq, prm, pl.grid, stream); break;
    case 64: e = run<64>(mp, mq, prm, pl.grid, stream); break;
    case 128: e = run<128>(mp, mq, prm, pl.grid, stream); break;
    case 256: e = run<256>(mp, mq, prm, pl.grid, stream); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  if (pl.splits > 1) {
    int64_t total = (int64_t)p_rows * q_rows;
    int blocks = (int)((total + 255) / 256);
    if (blocks > 4 * num_sms()) blocks = 4 * num_sms();
    splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(ws, pl.ws_ld, pl.splits, p_rows, q_rows, pl.swap,
                                                    static_cast<__nv_bfloat16*>(c), ldc);
    e = cudaGetLastError();
  }
  return e;
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
