// Paged attention over the KV pool: split-KV flash-decode and prefix-aware flash-prefill.
//
// Reference: nanovllm/layers/attention.py:303-375 calls flash_attn_varlen_func, reading
// the paged cache through block_table for prefix-hit prefill, chunked prefill and
// decode (q_len = 1); the torch fallback (:378-498) defines the semantics: causal mask
// offset by k_len - q_len, softmax scale 1/sqrt(D), GQA by repeating KV heads.
//
// Both kernels here read K/V straight from the paged pool [num_blocks, nkv, BS, 128]
// (bf16, or fp8 e4m3 with one scale per block per head), any power-of-two block size,
// and use bf16 mma.sync m16n8k16 tiles with fp32 accumulation (attention is a small
// share of the FLOPs here and decode is bandwidth-bound); tiles land in XOR-swizzled
// shared memory (conflict-free ldmatrix), by TMA for decode and cp.async for prefill.
//
// decode:  grid (splits, nkv, B).  Each CTA takes all G = nq/nkv query heads of one KV
//          head (packed as the 16 rows of one MMA tile) over one slice of the context.
//          A producer warp streams K/V tiles with TMA; 4 consumer warps split each
//          64-key tile.  With splits > 1 the CTA writes a normalised partial output and
//          its log2-sum-exp to scratch, and attn_combine merges the slices.
// prefill: grid (q tiles of 64, prefill seqs, nq).  4 warps x 16 query rows.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"

namespace nvb {

constexpr int AD = 128;        // head dim
constexpr int KTILE = 64;      // keys per tile
constexpr int ROWB = AD * 2;   // bytes per bf16 row
constexpr float LOG2E = 1.4426950408889634f;

__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * ROWB + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

struct AttnArgs {
  const __nv_bfloat16* q;   // [T, nq, 128]
  const void* k_cache;      // [NB, nkv, BS, 128]
  const void* v_cache;
  const float* k_scale;     // [NB, nkv] (fp8) or null
  const float* v_scale;
  const int* block_tables;  // [B, W]
  int W;
  const int* cu_q;          // [B + 1]
  const int* ctx_lens;      // [B]
  __nv_bfloat16* out;       // [T, nq, 128]
  float* part_o;            // [B, nq, splits, 128]
  float* part_lse;          // [B, nq, splits]
  int nq, nkv, block_size, num_blocks;
  int splits;
  int seq_offset;           // first sequence handled by this launch
  float scale_log2;
};

// Issue cp.async for one 64-key tile of K or V (head h of seq b) into `dst` (bf16:
// swizzled 64 x 256 B; fp8: plain 64 x 128 B staging).  Rows beyond k_len, or whose
// block id is out of range, are zero-filled.
template <bool FP8>
__device__ __forceinline__ void load_tile(const AttnArgs& a, const void* cache, int b, int h, int tile, int k_len,
                                          uint32_t dst) {
  const int* bt = a.block_tables + (int64_t)b * a.W;
  constexpr int CHUNKS = FP8 ? 8 : 16;  // 16-byte chunks per row
  constexpr int RB = FP8 ? AD : ROWB;
#pragma unroll
  for (int i = 0; i < KTILE * CHUNKS / 128; ++i) {
    int idx = threadIdx.x + i * 128;
    int r = idx / CHUNKS, c = idx % CHUNKS;
    int tok = tile * KTILE + r;
    bool valid = tok < k_len;
    const uint8_t* src = static_cast<const uint8_t*>(cache);
    if (valid) {
      int bi = tok / a.block_size;
      int blk = bi < a.W ? bt[bi] : -1;
      valid = blk >= 0 && blk < a.num_blocks;
      if (valid) src += ((((int64_t)blk * a.nkv + h) * a.block_size + (tok % a.block_size)) * RB) + c * 16;
    }
    uint32_t d = FP8 ? dst + r * RB + c * 16 : dst + swz(r, c);
    cp_async16(d, src, valid);
  }
}

// Per-row dequantisation scales of one 64-key tile into shared memory (threads 0..63).
__device__ __forceinline__ void tile_row_scales(const AttnArgs& a, const float* scales, int b, int h, int tile,
                                                int k_len, float* row_scale) {
  if (threadIdx.x < KTILE) {
    const int* bt = a.block_tables + (int64_t)b * a.W;
    const int tok = tile * KTILE + threadIdx.x;
    float s = 0.f;
    if (tok < k_len) {
      const int bi = tok / a.block_size;
      const int blk = bi < a.W ? bt[bi] : -1;
      if (blk >= 0 && blk < a.num_blocks) s = scales[(int64_t)blk * a.nkv + h];
    }
    row_scale[threadIdx.x] = s;
  }
}

// fp8 staging tile -> scaled bf16 swizzled tile (row scales from tile_row_scales).
__device__ __forceinline__ void convert_fp8_tile(const float* row_scale, const uint8_t* stage, uint8_t* dst) {
#pragma unroll
  for (int i = 0; i < KTILE * 16 / 128; ++i) {
    int idx = threadIdx.x + i * 128;
    int r = idx >> 4, c = idx & 15;
    const float s = row_scale[r];
    uint2 raw = *reinterpret_cast<const uint2*>(stage + r * AD + c * 8);
    float f[8];
    e4m3x4_to_f32(raw.x, f);
    e4m3x4_to_f32(raw.y, f + 4);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] *= s;
    *reinterpret_cast<uint4*>(dst + swz(r, c)) = f32_to_bf16x8(f);
  }
}

// ------------------------------------------------------------------------- decode
// Warp-specialised: warp 4 streams 64-key K/V tiles with TMA (128B swizzle) into a
// DSTAGES-deep ring; warps 0-3 each own 16 keys of every tile and keep their own
// online-softmax state, so consumers never wait on one another.  The last consumer
// warp to finish merges the four partial states (found with a shared-memory counter,
// no barrier).  Every mbarrier wait is time-bounded and reports through g_attn_error.
constexpr int DSTAGES = 3;
constexpr uint64_t ATT_WAIT_NS = 2000000000ull;

__device__ int g_attn_error = 0;

__device__ __forceinline__ bool att_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool att_wait(uint32_t bar, uint32_t parity, int code) {
  if (att_try(bar, parity)) return true;
  SpinBudget sb;
  while (!att_try(bar, parity)) {
    if (sb.expired(ATT_WAIT_NS)) {
      atomicCAS(&g_attn_error, 0, code);
      return false;
    }
  }
  return true;
}

struct DecodeArgs {
  AttnArgs a;
  int rows_per_box;  // min(64, block_size)
  int kv_fp8;
};

// Swizzled (TMA 128B pattern) bf16 tile: [2 halves of 64 dims][64 rows][128 B].
__device__ __forceinline__ uint32_t tswz(int r, int c16) {
  return (uint32_t)((c16 >> 3) * 8192 + r * 128 + ((((c16 & 7) ^ (r & 7))) << 4));
}

template <bool FP8>
__global__ void __launch_bounds__(160, 2)
    attn_decode_tma_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                           DecodeArgs da) {
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  const AttnArgs& a = da.a;
  extern __shared__ __align__(1024) uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  constexpr int KV_TILE = FP8 ? KTILE * AD : KTILE * ROWB;  // bytes of one K (or V) tile
  constexpr int STAGE = 2 * KV_TILE;
  uint8_t* conv = dsm + DSTAGES * STAGE;                          // fp8: per-warp bf16 staging 4 x 8 KB
  const int G = a.nq / a.nkv;
  uint8_t* comb = conv + (FP8 ? 4 * 8192 : 0);                    // combine: [4][G][128] f32 + [4][16][2] f32
  uint64_t* bars = reinterpret_cast<uint64_t*>(comb + 4 * G * AD * 4 + 4 * 16 * 2 * 4);
  int* done_ctr = reinterpret_cast<int*>(bars + 2 * DSTAGES);
  const uint32_t bar0 = smem_u32(bars);
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z + a.seq_offset;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int k_len = a.ctx_lens[b];
  const int qrow = a.cu_q[b];
  const int n_tiles = (k_len + KTILE - 1) / KTILE;
  const int per = (n_tiles + a.splits - 1) / a.splits;
  const int t0 = split * per;
  const int t1 = min(n_tiles, t0 + per);
  const int qh0 = h * G;

  if (t0 >= t1) {
    if (a.splits > 1) {
      for (int r = threadIdx.x; r < G; r += blockDim.x)
        a.part_lse[((int64_t)b * a.nq + qh0 + r) * a.splits + split] = -INFINITY;
    } else {
      for (int i = threadIdx.x; i < G * AD; i += blockDim.x)
        a.out[((int64_t)qrow * a.nq + qh0) * AD + i] = __float2bfloat16(0.f);
    }
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < DSTAGES; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8u * s));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 4;" ::"r"(bar0 + 8u * (DSTAGES + s)));
    }
    *done_ctr = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 4) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      const int* bt = a.block_tables + (int64_t)b * a.W;
      const int rpb = da.rows_per_box;
      const int nsub = KTILE / rpb;
      bool ok = true;
      int issued = 0;
      for (int t = t0; t < t1; ++t, ++issued) {
        const int i = t - t0, s = i % DSTAGES;
        const uint32_t round = i / DSTAGES;
        if (!att_wait(bar0 + 8u * (DSTAGES + s), (round & 1) ^ 1, 1)) {
          ok = false;
          break;
        }
        const uint32_t full = bar0 + 8u * s;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(full), "r"(STAGE) : "memory");
        const uint32_t kdst = smem_u32(dsm + s * STAGE), vdst = kdst + KV_TILE;
        for (int j = 0; j < nsub; ++j) {
          const int tok = t * KTILE + j * rpb;
          const int bi = tok / a.block_size;
          int blk = bi < a.W ? bt[bi] : 0;
          if (blk < 0 || blk >= a.num_blocks) blk = 0;
          const int row = (blk * a.nkv + h) * a.block_size + (tok % a.block_size);
          if (FP8) {
            const uint32_t off = j * rpb * AD;
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
                "[%2];" ::"r"(kdst + off), "l"(reinterpret_cast<uint64_t>(&kmap)), "r"(full), "r"(0), "r"(row)
                : "memory");
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
                "[%2];" ::"r"(vdst + off), "l"(reinterpret_cast<uint64_t>(&vmap)), "r"(full), "r"(0), "r"(row)
                : "memory");
          } else {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              const uint32_t off = half * 8192 + j * rpb * 128;
              asm volatile(
                  "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
                  "[%2];" ::"r"(kdst + off), "l"(reinterpret_cast<uint64_t>(&kmap)), "r"(full), "r"(half * 64),
                  "r"(row)
                  : "memory");
              asm volatile(
                  "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
                  "[%2];" ::"r"(vdst + off), "l"(reinterpret_cast<uint64_t>(&vmap)), "r"(full), "r"(half * 64),
                  "r"(row)
                  : "memory");
            }
          }
        }
      }
      // Do not leave while copies this thread issued may still be landing.
      const int n = issued < DSTAGES ? issued : DSTAGES;
      for (int i = issued - n; i < issued; ++i) {
        const uint32_t full = bar0 + 8u * (i % DSTAGES);
        SpinBudget sb;
        while (!att_try(full, (i / DSTAGES) & 1) && !sb.expired(ATT_WAIT_NS)) {
        }
      }
      (void)ok;
    }
    return;
  }

  // --------------------------------------------------------------- consumers
  // Q fragments straight from global memory (rows >= G are zero)
  uint32_t qf[8][4];
  {
    const int r0 = lane >> 2, r1 = r0 + 8;
    const __nv_bfloat16* q0p = a.q + ((int64_t)qrow * a.nq + qh0 + (r0 < G ? r0 : 0)) * AD;
    const __nv_bfloat16* q1p = a.q + ((int64_t)qrow * a.nq + qh0 + (r1 < G ? r1 : 0)) * AD;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int c = kk * 16 + (lane & 3) * 2;
      qf[kk][0] = r0 < G ? *reinterpret_cast<const uint32_t*>(q0p + c) : 0u;
      qf[kk][1] = r1 < G ? *reinterpret_cast<const uint32_t*>(q1p + c) : 0u;
      qf[kk][2] = r0 < G ? *reinterpret_cast<const uint32_t*>(q0p + c + 8) : 0u;
      qf[kk][3] = r1 < G ? *reinterpret_cast<const uint32_t*>(q1p + c + 8) : 0u;
    }
  }
  float acc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int* bt = a.block_tables + (int64_t)b * a.W;
  uint8_t* myconv = conv + warp * 8192;  // fp8 only: 2 x [16 rows][256 B]

  for (int t = t0; t < t1; ++t) {
    const int i = t - t0, s = i % DSTAGES;
    if (!att_wait(bar0 + 8u * s, (i / DSTAGES) & 1, 2)) break;
    const uint8_t* kt = dsm + s * STAGE;
    const uint8_t* vt = kt + KV_TILE;
    uint32_t kb, vb;  // ldmatrix bases; rows are addressed as warp-local 0..15 (+ warp*16 for TMA tiles)
    int rbase;
    if (FP8) {
      // dequantise this warp's 16 K rows and 16 V rows into its bf16 staging (row 256 B, xor
      // swizzle).  The 16 rows lie in one block (block_size >= 16), so one scale pair serves all.
      float ksc = 0.f, vsc = 0.f;
      if (lane == 0) {
        const int bi = (t * KTILE + warp * 16) / a.block_size;
        int blk = bi < a.W ? bt[bi] : 0;
        if (blk < 0 || blk >= a.num_blocks) blk = 0;
        ksc = a.k_scale[(int64_t)blk * a.nkv + h];
        vsc = a.v_scale[(int64_t)blk * a.nkv + h];
      }
      ksc = __shfl_sync(FULL_MASK, ksc, 0);
      vsc = __shfl_sync(FULL_MASK, vsc, 0);
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int idx = lane + it * 32;       // 0..127 -> (row 0..15, 16-byte fp8 chunk 0..7)
        const int r = idx >> 3, c = idx & 7;
        const int gr = warp * 16 + r;
        const uint32_t soff = gr * 128 + ((c ^ (gr & 7)) << 4);
        const uint4 kr = *reinterpret_cast<const uint4*>(kt + soff);
        const uint4 vr = *reinterpret_cast<const uint4*>(vt + soff);
        float f[16];
        e4m3x4_to_f32(kr.x, f); e4m3x4_to_f32(kr.y, f + 4); e4m3x4_to_f32(kr.z, f + 8); e4m3x4_to_f32(kr.w, f + 12);
#pragma unroll
        for (int j = 0; j < 16; ++j) f[j] *= ksc;
        *reinterpret_cast<uint4*>(myconv + swz(r, 2 * c)) = f32_to_bf16x8(f);
        *reinterpret_cast<uint4*>(myconv + swz(r, 2 * c + 1)) = f32_to_bf16x8(f + 8);
        e4m3x4_to_f32(vr.x, f); e4m3x4_to_f32(vr.y, f + 4); e4m3x4_to_f32(vr.z, f + 8); e4m3x4_to_f32(vr.w, f + 12);
#pragma unroll
        for (int j = 0; j < 16; ++j) f[j] *= vsc;
        *reinterpret_cast<uint4*>(myconv + 4096 + swz(r, 2 * c)) = f32_to_bf16x8(f);
        *reinterpret_cast<uint4*>(myconv + 4096 + swz(r, 2 * c + 1)) = f32_to_bf16x8(f + 8);
      }
      __syncwarp();
      // the fp8 stage is no longer needed by this warp
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar0 + 8u * (DSTAGES + s)) : "memory");
      kb = smem_u32(myconv);
      vb = kb + 4096;
      rbase = 0;
    } else {
      kb = smem_u32(kt);
      vb = smem_u32(vt);
      rbase = warp * 16;
    }
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t b0, b1, b2, b3;
      const int r = rbase + (lane & 7) + ((lane >> 4) << 3), c = kk * 2 + ((lane >> 3) & 1);
      ldsm_x4(kb + (FP8 ? swz(r, c) : tswz(r, c)), b0, b1, b2, b3);
      mma_bf16(sc[0], qf[kk], b0, b1);
      mma_bf16(sc[1], qf[kk], b2, b3);
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = t * KTILE + warp * 16 + nt * 8 + (lane & 3) * 2 + e;
        const bool ok = key < k_len;
        sc[nt][e] = ok ? sc[nt][e] * a.scale_log2 : -INFINITY;
        sc[nt][2 + e] = ok ? sc[nt][2 + e] * a.scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, sc[nt][e]);
        mx1 = fmaxf(mx1, sc[nt][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(FULL_MASK, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(FULL_MASK, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(FULL_MASK, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(FULL_MASK, mx1, 2));
    const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
    const float base0 = nm0 == -INFINITY ? 0.f : nm0, base1 = nm1 == -INFINITY ? 0.f : nm1;
    const float al0 = exp2f(m0 - base0), al1 = exp2f(m1 - base1);
    m0 = nm0;
    m1 = nm1;
    float p[2][4];
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      p[nt][0] = exp2f(sc[nt][0] - base0);
      p[nt][1] = exp2f(sc[nt][1] - base0);
      p[nt][2] = exp2f(sc[nt][2] - base1);
      p[nt][3] = exp2f(sc[nt][3] - base1);
      rs0 += p[nt][0] + p[nt][1];
      rs1 += p[nt][2] + p[nt][3];
    }
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      acc[j][0] *= al0;
      acc[j][1] *= al0;
      acc[j][2] *= al1;
      acc[j][3] *= al1;
    }
    const uint32_t pa[4] = {pack_bf16(p[0][0], p[0][1]), pack_bf16(p[0][2], p[0][3]), pack_bf16(p[1][0], p[1][1]),
                            pack_bf16(p[1][2], p[1][3])};
#pragma unroll
    for (int np = 0; np < 8; ++np) {
      uint32_t b0, b1, b2, b3;
      const int r = rbase + (lane & 7) + ((lane >> 3) & 1) * 8, c = np * 2 + (lane >> 4);
      ldsm_x4_t(vb + (FP8 ? swz(r, c) : tswz(r, c)), b0, b1, b2, b3);
      mma_bf16(acc[2 * np], pa, b0, b1);
      mma_bf16(acc[2 * np + 1], pa, b2, b3);
    }
    if (!FP8) {
      __syncwarp();
      if (lane == 0)
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar0 + 8u * (DSTAGES + s)) : "memory");
    } else {
      __syncwarp();  // staging is rewritten next tile
    }
  }

  // publish this warp's state; the last warp to arrive merges all four
  l0 += __shfl_xor_sync(FULL_MASK, l0, 1);
  l0 += __shfl_xor_sync(FULL_MASK, l0, 2);
  l1 += __shfl_xor_sync(FULL_MASK, l1, 1);
  l1 += __shfl_xor_sync(FULL_MASK, l1, 2);
  float* sm_acc = reinterpret_cast<float*>(comb);
  float* sm_ml = sm_acc + 4 * G * AD;
  const int r0 = lane >> 2, r1 = r0 + 8;
  if ((lane & 3) == 0) {
    sm_ml[(warp * 16 + r0) * 2] = m0;
    sm_ml[(warp * 16 + r0) * 2 + 1] = l0;
    sm_ml[(warp * 16 + r1) * 2] = m1;
    sm_ml[(warp * 16 + r1) * 2 + 1] = l1;
  }
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int c = nt * 8 + (lane & 3) * 2;
    if (r0 < G) *reinterpret_cast<float2*>(sm_acc + (warp * G + r0) * AD + c) = make_float2(acc[nt][0], acc[nt][1]);
    if (r1 < G) *reinterpret_cast<float2*>(sm_acc + (warp * G + r1) * AD + c) = make_float2(acc[nt][2], acc[nt][3]);
  }
  __threadfence_block();
  __syncwarp();
  int last = 0;
  if (lane == 0) last = atomicAdd(done_ctr, 1) == 3;
  last = __shfl_sync(FULL_MASK, last, 0);
  if (!last) return;
  __threadfence_block();
  for (int i = lane; i < G * AD; i += 32) {
    const int r = i / AD, c = i % AD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_ml[(w * 16 + r) * 2]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(sm_ml[(w * 16 + r) * 2] - M);
        L += sm_ml[(w * 16 + r) * 2 + 1] * f;
        O += sm_acc[(w * G + r) * AD + c] * f;
      }
    }
    const float o = L > 0.f ? O / L : 0.f;
    if (a.splits == 1) {
      a.out[((int64_t)qrow * a.nq + qh0 + r) * AD + c] = __float2bfloat16(o);
    } else {
      const int64_t pi = ((int64_t)b * a.nq + qh0 + r) * a.splits + split;
      a.part_o[pi * AD + c] = o;
      if (c == 0) a.part_lse[pi] = L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
}

// fp8 decode with the keys on the MMA's M side.  S^T[16 keys x 8 heads] = K Q^T and
// O^T[16 dims x 8 heads] += V^T P^T, f16 tensor-core inputs, fp32 accumulators.  The fp8
// bytes go from shared memory straight into MMA fragments (one cvt.f16x2.e4m3x2 per two
// values; no staging copy): the reduction dimension of both products may be permuted
// freely, so a thread's K fragment is 32 contiguous bytes of one key row (dims 32c..32c+31
// for lane%4 = c, Q loaded in the same order) and its V fragment 16 contiguous bytes of
// four key rows (output dims 16r..16r+15 for lane/4 = r); P^T goes from the S^T
// accumulator to the B operand with two movmatrix transposes.  Scales: K's folds into the
// score multiplier; V's is applied by keeping the accumulator in units of the current
// tile's scale (the online-softmax rescale absorbs the ratio between tiles).  G <= 8,
// block_size >= 16 (a warp's 16 keys then share one block and one scale pair).
__device__ __forceinline__ void mma_f16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Two e4m3 pairs (the low and high 16 bits of x) -> two f16x2 words.
__device__ __forceinline__ void e4m3x2x2_to_f16x2(uint32_t x, uint32_t& lo, uint32_t& hi) {
  asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n cvt.rn.f16x2.e4m3x2 %0, l;\n cvt.rn.f16x2.e4m3x2 %1, h;\n}\n"
      : "=r"(lo), "=r"(hi)
      : "r"(x));
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(x));
  return d;
}
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %2, %1;" : "=r"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

__global__ void __launch_bounds__(160, 3)
    attn_decode_fp8_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                           DecodeArgs da) {
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  const AttnArgs& a = da.a;
  extern __shared__ __align__(1024) uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  constexpr int KV_TILE = KTILE * AD;
  constexpr int STAGE = 2 * KV_TILE;
  const int G = a.nq / a.nkv;
  uint8_t* comb = dsm + DSTAGES * STAGE;  // [4][G][128] f32 + [4][16][2] f32
  uint64_t* bars = reinterpret_cast<uint64_t*>(comb + 4 * G * AD * 4 + 4 * 16 * 2 * 4);
  int* done_ctr = reinterpret_cast<int*>(bars + 2 * DSTAGES);
  const uint32_t bar0 = smem_u32(bars);
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z + a.seq_offset;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int k_len = a.ctx_lens[b];
  const int qrow = a.cu_q[b];
  const int n_tiles = (k_len + KTILE - 1) / KTILE;
  const int per = (n_tiles + a.splits - 1) / a.splits;
  const int t0 = split * per;
  const int t1 = min(n_tiles, t0 + per);
  const int qh0 = h * G;

  if (t0 >= t1) {
    if (a.splits > 1) {
      for (int r = threadIdx.x; r < G; r += blockDim.x)
        a.part_lse[((int64_t)b * a.nq + qh0 + r) * a.splits + split] = -INFINITY;
    } else {
      for (int i = threadIdx.x; i < G * AD; i += blockDim.x)
        a.out[((int64_t)qrow * a.nq + qh0) * AD + i] = __float2bfloat16(0.f);
    }
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < DSTAGES; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8u * s));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 4;" ::"r"(bar0 + 8u * (DSTAGES + s)));
    }
    *done_ctr = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 4) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      const int* bt = a.block_tables + (int64_t)b * a.W;
      const int rpb = da.rows_per_box;
      const int nsub = KTILE / rpb;
      int issued = 0;
      for (int t = t0; t < t1; ++t, ++issued) {
        const int i = t - t0, s = i % DSTAGES;
        if (!att_wait(bar0 + 8u * (DSTAGES + s), ((i / DSTAGES) & 1) ^ 1, 3)) break;
        const uint32_t full = bar0 + 8u * s;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(full), "r"(STAGE) : "memory");
        const uint32_t kdst = smem_u32(dsm + s * STAGE), vdst = kdst + KV_TILE;
        for (int j = 0; j < nsub; ++j) {
          const int tok = t * KTILE + j * rpb;
          const int bi = tok / a.block_size;
          int blk = bi < a.W ? bt[bi] : 0;
          if (blk < 0 || blk >= a.num_blocks) blk = 0;
          const int row = (blk * a.nkv + h) * a.block_size + (tok % a.block_size);
          const uint32_t off = j * rpb * AD;
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
              "[%2];" ::"r"(kdst + off), "l"(reinterpret_cast<uint64_t>(&kmap)), "r"(full), "r"(0), "r"(row)
              : "memory");
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
              "[%2];" ::"r"(vdst + off), "l"(reinterpret_cast<uint64_t>(&vmap)), "r"(full), "r"(0), "r"(row)
              : "memory");
        }
      }
      // Do not leave while copies this thread issued may still be landing.
      const int n = issued < DSTAGES ? issued : DSTAGES;
      for (int i = issued - n; i < issued; ++i) {
        const uint32_t full = bar0 + 8u * (i % DSTAGES);
        SpinBudget sb;
        while (!att_try(full, (i / DSTAGES) & 1) && !sb.expired(ATT_WAIT_NS)) {
        }
      }
    }
    return;
  }

  // --------------------------------------------------------------- consumers
  const int r = lane >> 2, c = lane & 3;
  // Q^T fragments (B operand): head r, dims 32c + 4kk + {0,1} and {2,3}; heads >= G are zero
  uint32_t qf[8][2];
  {
    const __nv_bfloat16* qp = a.q + ((int64_t)qrow * a.nq + qh0 + (r < G ? r : 0)) * AD + 32 * c;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 v = r < G ? *reinterpret_cast<const uint4*>(qp + 8 * i) : make_uint4(0, 0, 0, 0);
      float f[8];
      bf16x8_to_f32(v, f);
      qf[2 * i][0] = pack_f16(f[0], f[1]);
      qf[2 * i][1] = pack_f16(f[2], f[3]);
      qf[2 * i + 1][0] = pack_f16(f[4], f[5]);
      qf[2 * i + 1][1] = pack_f16(f[6], f[7]);
    }
  }
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f, vsc_run = 1.f;
  const int* bt = a.block_tables + (int64_t)b * a.W;
  const int kr0 = warp * 16 + r, kr1 = kr0 + 8;       // this thread's K rows in the tile
  const int vr = warp * 16 + 2 * c;                   // V rows vr, vr+1, vr+8, vr+9

  for (int t = t0; t < t1; ++t) {
    const int i = t - t0, s = i % DSTAGES;
    if (!att_wait(bar0 + 8u * s, (i / DSTAGES) & 1, 4)) break;
    const uint8_t* kt = dsm + s * STAGE;
    const uint8_t* vt = kt + KV_TILE;
    // K: bytes [32c, 32c + 32) of rows kr0 and kr1 (TMA 128-byte swizzle: chunk ^ (row & 7))
    const uint4 ka0 = *reinterpret_cast<const uint4*>(kt + kr0 * AD + (((2 * c) ^ (kr0 & 7)) << 4));
    const uint4 ka1 = *reinterpret_cast<const uint4*>(kt + kr0 * AD + (((2 * c + 1) ^ (kr0 & 7)) << 4));
    const uint4 kb0 = *reinterpret_cast<const uint4*>(kt + kr1 * AD + (((2 * c) ^ (kr1 & 7)) << 4));
    const uint4 kb1 = *reinterpret_cast<const uint4*>(kt + kr1 * AD + (((2 * c + 1) ^ (kr1 & 7)) << 4));
    // V: bytes [16r, 16r + 16) of rows vr, vr+1, vr+8, vr+9
    uint4 v0 = *reinterpret_cast<const uint4*>(vt + vr * AD + ((r ^ (vr & 7)) << 4));
    uint4 v1 = *reinterpret_cast<const uint4*>(vt + (vr + 1) * AD + ((r ^ ((vr + 1) & 7)) << 4));
    uint4 v2 = *reinterpret_cast<const uint4*>(vt + (vr + 8) * AD + ((r ^ ((vr + 8) & 7)) << 4));
    uint4 v3 = *reinterpret_cast<const uint4*>(vt + (vr + 9) * AD + ((r ^ ((vr + 9) & 7)) << 4));
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar0 + 8u * (DSTAGES + s)) : "memory");
    const int key0 = t * KTILE + warp * 16;
    if (key0 + 16 > k_len) {
      // rows past the context may hold any bytes (an e4m3 NaN included): zero them
      const uint4 z = make_uint4(0, 0, 0, 0);
      if (key0 + 2 * c >= k_len) v0 = z;
      if (key0 + 2 * c + 1 >= k_len) v1 = z;
      if (key0 + 2 * c + 8 >= k_len) v2 = z;
      if (key0 + 2 * c + 9 >= k_len) v3 = z;
    }
    float ksc = 0.f, vsc = 0.f;
    if (lane == 0) {
      const int bi = key0 / a.block_size;
      int blk = bi < a.W ? bt[bi] : 0;
      if (blk < 0 || blk >= a.num_blocks) blk = 0;
      ksc = a.k_scale[(int64_t)blk * a.nkv + h];
      vsc = a.v_scale[(int64_t)blk * a.nkv + h];
    }
    ksc = __shfl_sync(FULL_MASK, ksc, 0);
    vsc = __shfl_sync(FULL_MASK, vsc, 0);

    // S^T = K Q^T over 8 steps of 16 (permuted) dims
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t w0 = word_of(kk < 4 ? ka0 : ka1, kk & 3), w1 = word_of(kk < 4 ? kb0 : kb1, kk & 3);
      uint32_t af[4];
      e4m3x2x2_to_f16x2(w0, af[0], af[2]);
      e4m3x2x2_to_f16x2(w1, af[1], af[3]);
      mma_f16(sc, af, qf[kk][0], qf[kk][1]);
    }
    // online softmax per head (columns 2c, 2c+1); rows are keys kr0 (sc[0..1]) and kr1 (sc[2..3])
    const float mul = ksc * a.scale_log2;
    const bool ok0 = key0 + r < k_len, ok1 = key0 + r + 8 < k_len;
    sc[0] = ok0 ? sc[0] * mul : -INFINITY;
    sc[1] = ok0 ? sc[1] * mul : -INFINITY;
    sc[2] = ok1 ? sc[2] * mul : -INFINITY;
    sc[3] = ok1 ? sc[3] * mul : -INFINITY;
    float mx0 = fmaxf(sc[0], sc[2]), mx1 = fmaxf(sc[1], sc[3]);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(FULL_MASK, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(FULL_MASK, mx1, o));
    }
    const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
    const float base0 = nm0 == -INFINITY ? 0.f : nm0, base1 = nm1 == -INFINITY ? 0.f : nm1;
    const float al0 = exp2f(m0 - base0), al1 = exp2f(m1 - base1);
    m0 = nm0;
    m1 = nm1;
    const float p0 = exp2f(sc[0] - base0), p1 = exp2f(sc[1] - base1);
    const float p2 = exp2f(sc[2] - base0), p3 = exp2f(sc[3] - base1);
    l0 = l0 * al0 + p0 + p2;
    l1 = l1 * al1 + p1 + p3;
    // the accumulator is kept in units of the current tile's V scale
    const float ratio = vsc_run / vsc;
    vsc_run = vsc;
    const float f0 = al0 * ratio, f1 = al1 * ratio;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      acc[u][0] *= f0;
      acc[u][1] *= f1;
      acc[u][2] *= f0;
      acc[u][3] *= f1;
    }
    // P^T as the B operand: transpose the [key][head] f16 pairs
    const uint32_t pb0 = movmatrix_t(pack_f16(p0, p1));
    const uint32_t pb1 = movmatrix_t(pack_f16(p2, p3));
    // O^T += V^T P^T over 8 tiles of 16 output dims (dims 16r + 2u, 16r + 2u + 1)
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const uint32_t sel = (u & 1) ? 0x7362u : 0x5140u;
      const uint32_t x = prmt(word_of(v0, u >> 1), word_of(v1, u >> 1), sel);
      const uint32_t y = prmt(word_of(v2, u >> 1), word_of(v3, u >> 1), sel);
      uint32_t af[4];
      e4m3x2x2_to_f16x2(x, af[0], af[1]);
      e4m3x2x2_to_f16x2(y, af[2], af[3]);
      mma_f16(acc[u], af, pb0, pb1);
    }
  }

  // publish this warp's state; the last warp to arrive merges all four
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l0 += __shfl_xor_sync(FULL_MASK, l0, o);
    l1 += __shfl_xor_sync(FULL_MASK, l1, o);
  }
  float* sm_acc = reinterpret_cast<float*>(comb);
  float* sm_ml = sm_acc + 4 * G * AD;
  const int h0 = 2 * c, h1 = 2 * c + 1;
  if (r == 0) {
    sm_ml[(warp * 16 + h0) * 2] = m0;
    sm_ml[(warp * 16 + h0) * 2 + 1] = l0;
    sm_ml[(warp * 16 + h1) * 2] = m1;
    sm_ml[(warp * 16 + h1) * 2 + 1] = l1;
  }
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    if (h0 < G)
      *reinterpret_cast<float2*>(sm_acc + (warp * G + h0) * AD + 16 * r + 2 * u) =
          make_float2(acc[u][0] * vsc_run, acc[u][2] * vsc_run);
    if (h1 < G)
      *reinterpret_cast<float2*>(sm_acc + (warp * G + h1) * AD + 16 * r + 2 * u) =
          make_float2(acc[u][1] * vsc_run, acc[u][3] * vsc_run);
  }
  __threadfence_block();
  __syncwarp();
  int last = 0;
  if (lane == 0) last = atomicAdd(done_ctr, 1) == 3;
  last = __shfl_sync(FULL_MASK, last, 0);
  if (!last) return;
  __threadfence_block();
  for (int i = lane; i < G * AD; i += 32) {
    const int hh = i / AD, d = i % AD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_ml[(w * 16 + hh) * 2]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(sm_ml[(w * 16 + hh) * 2] - M);
        L += sm_ml[(w * 16 + hh) * 2 + 1] * f;
        O += sm_acc[(w * G + hh) * AD + d] * f;
      }
    }
    const float o = L > 0.f ? O / L : 0.f;
    if (a.splits == 1) {
      a.out[((int64_t)qrow * a.nq + qh0 + hh) * AD + d] = __float2bfloat16(o);
    } else {
      const int64_t pi = ((int64_t)b * a.nq + qh0 + hh) * a.splits + split;
      a.part_o[pi * AD + d] = o;
      if (d == 0) a.part_lse[pi] = L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
}

// Merge split partials: one CTA per (seq, q head), one thread per dim.
__global__ void attn_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                    const int* __restrict__ cu_q, __nv_bfloat16* __restrict__ out, int nq, int splits,
                                    int seq_offset) {
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  const int bh = blockIdx.x;
  const int b = bh / nq + seq_offset, hq = bh % nq;
  const int64_t base = ((int64_t)b * nq + hq) * splits;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_lse[base + s]);
  float L = 0.f, O = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      // An empty split (no keys) writes only its -inf log-sum-exp, never its output row:
      // skip it, so stale scratch (possibly NaN) never meets a zero weight.
      const float lse = part_lse[base + s];
      if (lse == -INFINITY) continue;
      const float w = exp2f(lse - M);
      L += w;
      O += w * part_o[(base + s) * AD + threadIdx.x];
    }
  }
  out[((int64_t)cu_q[b] * nq + hq) * AD + threadIdx.x] = __float2bfloat16(L > 0.f ? O / L : 0.f);
}

// ------------------------------------------------------------------------ prefill
template <bool FP8>
__global__ void __launch_bounds__(128) attn_prefill_kernel(AttnArgs a) {
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sq = smem;                      // 64 x 256 B
  uint8_t* sk = smem + KTILE * ROWB;       // 2 x 64 x 256
  uint8_t* sv = sk + 2 * KTILE * ROWB;     // 2 x 64 x 256
  uint8_t* stg = sv + 2 * KTILE * ROWB;    // fp8 staging 4 x 64 x 128
  const int b = blockIdx.y + a.seq_offset;
  const int hq = blockIdx.z;
  const int G = a.nq / a.nkv;
  const int h = hq / G;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int qs = a.cu_q[b];
  const int q_len = a.cu_q[b + 1] - qs;
  const int row0 = blockIdx.x * 64;
  if (row0 >= q_len) return;
  const int k_len = a.ctx_lens[b];
  const int off = k_len - q_len;
  const int kmax = min(k_len, off + row0 + 64);
  const int n_tiles = (kmax + KTILE - 1) / KTILE;

  for (int idx = threadIdx.x; idx < 64 * 16; idx += 128) {
    int r = idx >> 4, c = idx & 15;
    bool v = row0 + r < q_len;
    const __nv_bfloat16* src = a.q + ((int64_t)(qs + row0 + (v ? r : 0)) * a.nq + hq) * AD + c * 8;
    cp_async16(smem_u32(sq) + swz(r, c), src, v);
  }
  auto issue = [&](int tile, int st) {
    if (FP8) {
      load_tile<true>(a, a.k_cache, b, h, tile, k_len, smem_u32(stg) + st * KTILE * AD);
      load_tile<true>(a, a.v_cache, b, h, tile, k_len, smem_u32(stg) + (2 + st) * KTILE * AD);
    } else {
      load_tile<false>(a, a.k_cache, b, h, tile, k_len, smem_u32(sk) + st * KTILE * ROWB);
      load_tile<false>(a, a.v_cache, b, h, tile, k_len, smem_u32(sv) + st * KTILE * ROWB);
    }
  };
  if (n_tiles > 0) issue(0, 0);
  cp_commit();

  const int qr0 = warp * 16 + (lane >> 2);        // local rows of this thread
  const int qpos0 = off + row0 + qr0, qpos1 = qpos0 + 8;
  uint32_t qf[8][4];
  float acc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  bool q_loaded = false;

  for (int t = 0; t < n_tiles; ++t) {
    const int st = t & 1;
    if (t + 1 < n_tiles) {
      issue(t + 1, st ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    int cs = st;
    if (FP8) {
      __shared__ float ks_row[KTILE], vs_row[KTILE];
      tile_row_scales(a, a.k_scale, b, h, t, k_len, ks_row);
      tile_row_scales(a, a.v_scale, b, h, t, k_len, vs_row);
      __syncthreads();
      convert_fp8_tile(ks_row, stg + st * KTILE * AD, sk);
      convert_fp8_tile(vs_row, stg + (2 + st) * KTILE * AD, sv);
      __syncthreads();
      cs = 0;
    }
    if (!q_loaded) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = kk * 2 + (lane >> 4);
        ldsm_x4(smem_u32(sq) + swz(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
      q_loaded = true;
    }
    const uint32_t kb = smem_u32(sk) + cs * KTILE * ROWB;
    const uint32_t vb = smem_u32(sv) + cs * KTILE * ROWB;
    // Skip tiles entirely above this warp's diagonal (still joins the barriers).
    const bool warp_active = t * KTILE <= off + row0 + warp * 16 + 15;
    if (warp_active) {
      float s[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b0, b1, b2, b3;
          int r = np * 16 + (lane & 7) + ((lane >> 4) << 3), c = kk * 2 + ((lane >> 3) & 1);
          ldsm_x4(kb + swz(r, c), b0, b1, b2, b3);
          mma_bf16(s[2 * np], qf[kk], b0, b1);
          mma_bf16(s[2 * np + 1], qf[kk], b2, b3);
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          int key = t * KTILE + nt * 8 + (lane & 3) * 2 + e;
          bool ok0 = key < k_len && key <= qpos0;
          bool ok1 = key < k_len && key <= qpos1;
          s[nt][e] = ok0 ? s[nt][e] * a.scale_log2 : -INFINITY;
          s[nt][2 + e] = ok1 ? s[nt][2 + e] * a.scale_log2 : -INFINITY;
          mx0 = fmaxf(mx0, s[nt][e]);
          mx1 = fmaxf(mx1, s[nt][2 + e]);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(FULL_MASK, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(FULL_MASK, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(FULL_MASK, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(FULL_MASK, mx1, 2));
      const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
      const float base0 = nm0 == -INFINITY ? 0.f : nm0, base1 = nm1 == -INFINITY ? 0.f : nm1;
      const float al0 = exp2f(m0 - base0), al1 = exp2f(m1 - base1);
      m0 = nm0;
      m1 = nm1;
      float rs0 = 0.f, rs1 = 0.f;
      uint32_t pa[4][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        float p0 = exp2f(s[nt][0] - base0), p1 = exp2f(s[nt][1] - base0);
        float p2 = exp2f(s[nt][2] - base1), p3 = exp2f(s[nt][3] - base1);
        rs0 += p0 + p1;
        rs1 += p2 + p3;
        // A fragment of P for key step nt/2: regs (nt even) 0,1 / (nt odd) 2,3
        pa[nt >> 1][(nt & 1) * 2] = pack_bf16(p0, p1);
        pa[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16(p2, p3);
      }
      l0 = l0 * al0 + rs0;
      l1 = l1 * al1 + rs1;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        acc[i][0] *= al0;
        acc[i][1] *= al0;
        acc[i][2] *= al1;
        acc[i][3] *= al1;
      }
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          uint32_t b0, b1, b2, b3;
          int r = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = np * 2 + (lane >> 4);
          ldsm_x4_t(vb + swz(r, c), b0, b1, b2, b3);
          mma_bf16(acc[2 * np], pa[ks], b0, b1);
          mma_bf16(acc[2 * np + 1], pa[ks], b2, b3);
        }
      }
    }
    __syncthreads();
  }
  l0 += __shfl_xor_sync(FULL_MASK, l0, 1);
  l0 += __shfl_xor_sync(FULL_MASK, l0, 2);
  l1 += __shfl_xor_sync(FULL_MASK, l1, 1);
  l1 += __shfl_xor_sync(FULL_MASK, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int gr0 = row0 + qr0, gr1 = gr0 + 8;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    int c = nt * 8 + (lane & 3) * 2;
    if (gr0 < q_len)
      *reinterpret_cast<uint32_t*>(a.out + ((int64_t)(qs + gr0) * a.nq + hq) * AD + c) =
          pack_bf16(acc[nt][0] * inv0, acc[nt][1] * inv0);
    if (gr1 < q_len)
      *reinterpret_cast<uint32_t*>(a.out + ((int64_t)(qs + gr1) * a.nq + hq) * AD + c) =
          pack_bf16(acc[nt][2] * inv1, acc[nt][3] * inv1);
  }
}

static int prefill_smem(bool fp8) { return KTILE * ROWB + 4 * KTILE * ROWB + (fp8 ? 4 * KTILE * AD : 0); }

int attn_decode_splits(int num_seqs, int nkv, int max_ctx, int num_sms) {
  int ctas = num_seqs * nkv;
  int want = (2 * num_sms + ctas - 1) / ctas;
  int max_tiles = (max_ctx + KTILE - 1) / KTILE;
  int s = want < max_tiles ? want : max_tiles;
  if (s > 64) s = 64;
  return s < 1 ? 1 : s;
}

static PFN_cuTensorMapEncodeTiled_v12000 attn_encode() {
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

// ------------------------------------------------------------- prefill on tcgen05
// Prefix-aware causal flash-attention prefill on the 5th-generation tensor cores (bf16 KV).
//
// One CTA per (query tile, KV head, sequence).  GQA is packed into the MMA's 128 rows: row
// r holds query token t0 + r / G of query head h G + r % G, so the G heads that share a KV
// head share every K/V tile a CTA loads (G = nq / nkv, 128 / G tokens per tile).  Per 128-key
// tile j:
//   S_j = Q K_j^T      tcgen05.mma, A = Q (smem, K-major), B = K_j (smem, K-major), D in TMEM
//   P_j = exp2(S_j - m) softmax warps: one TMEM lane (= one row) per thread, no shuffles;
//                      P_j is written back into TMEM over S_j as packed bf16
//   O  += P_j V_j      tcgen05.mma, A = P_j (TMEM), B = V_j (smem, MN-major), D = O in TMEM
// S is double-buffered in TMEM (S_{j+1} runs on the tensor cores while the softmax warps
// work on S_j); K and V stream through a 2-stage TMA ring straight from the paged pool
// (one box per KV block, out-of-range blocks read as zeros).  The running maximum m is only
// raised, and O rescaled, when a row's maximum grows by more than 8 (a factor 256 in P,
// harmless in fp32 / bf16), so most tiles skip the rescale.
// Warps: 0 TMA producer, 1 TMEM allocator + MMA issuer, 2-5 softmax / correction / output.
// Every mbarrier wait is time-bounded (error word g_attn_error, codes 40-49).
namespace pf {

constexpr int TQ_ROWS = 128;  // MMA M: (query token, query head) rows per CTA
constexpr int TK = 128;       // keys per tile (MMA N of S, K of P V)
constexpr int NSTAGE = 2;     // K/V ring depth
constexpr int THREADS = 320;  // 10 warps: TMA, MMA, 8 softmax (two per TMEM lane quarter)
constexpr int HALF = TQ_ROWS * 64 * 2;  // bytes of one 64-dim half of a 128-row tile (16 KB)
constexpr int TILE = 2 * HALF;          // 32 KB: a 128 x 128 bf16 tile
constexpr float RESCALE_LOG2 = 8.f;

struct Args {
  const int* block_tables;
  int W;
  const int* cu_q;
  const int* ctx_lens;
  __nv_bfloat16* out;
  int nq, nkv, G, block_size, num_blocks, seq_offset;
  int kv_box;       // rows per K/V TMA box: min(block_size, 128)
  int kv_rows;      // rows of the 2-D [NB * nkv * BS, 128] pool view (an out-of-range row start)
  int qtiles;       // query tiles of the longest sequence of the launch
  int num_seqs;     // sequences of the launch (from seq_offset)
  float scale_log2;
};

__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tma2d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma3d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// D (TMEM) (+)= A (smem descriptor) * B (smem descriptor)
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// D (TMEM) (+)= A (TMEM) * B (smem descriptor)
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
// Shared-memory matrix descriptor, 128-byte swizzle, version 1 (sm_100).  K-major operands:
// 8-row groups 1024 B apart (sbo), lbo unused.  MN-major operands: lbo = distance between
// 64-element blocks along M/N, sbo = distance between 8-row groups along K.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
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
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// bf16 x bf16 -> f32, M = 128, N = 128; `b_mn_major`: B stored MN-major (V).
__device__ __forceinline__ constexpr uint32_t idesc(bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn_major ? (1u << 16) : 0u) | ((uint32_t)(128 >> 3) << 17) |
         ((uint32_t)(128 >> 4) << 24);
}

// TMEM columns: S buffers at 0 and 128, O buffers at 256 and 384.
__device__ __forceinline__ constexpr uint32_t s_col(int s) { return s ? 128u : 0u; }
__device__ __forceinline__ constexpr uint32_t o_col(int s) { return s ? 384u : 256u; }

}  // namespace pf

// 320 threads: one SM sub-partition holds three of the ten warps, so a thread gets at most 168
// of the sub-partition's 16 K registers (the launch bound lets ptxas plan for that)
__global__ void __launch_bounds__(pf::THREADS, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap, pf::Args a) {
  // Persistent: one CTA per SM walks the (query tile, KV head, sequence) items round-robin,
  // heaviest (latest) query tiles first.  Barrier phases and the K/V ring, S buffers and the
  // P V completion count run on CTA-wide counters across items; O is double-buffered in TMEM
  // so the softmax warps store one item's output while the MMAs of the next item run.
  using namespace pf;
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  extern __shared__ __align__(1024) uint8_t pf_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pf_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = sm;                           // Q: [2 halves][128 rows][128 B]
  uint8_t* sk = sq + TILE;                    // K ring: NSTAGE x TILE
  uint8_t* sv = sk + NSTAGE * TILE;           // V ring: NSTAGE x TILE
  uint64_t* bars = reinterpret_cast<uint64_t*>(sv + NSTAGE * TILE);
  // bars: q_full, q_empty, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], p_ready[2], s_free[2],
  //       o_done, o_final[2], o_empty[2], drain
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 23);
  const uint32_t b0 = smem_u32(bars);
  const uint32_t q_full = b0, q_empty = b0 + 8u;
  auto k_full = [&](int s) { return b0 + 8u * (2 + s); };
  auto k_empty = [&](int s) { return b0 + 8u * (4 + s); };
  auto v_full = [&](int s) { return b0 + 8u * (6 + s); };
  auto v_empty = [&](int s) { return b0 + 8u * (8 + s); };
  auto s_full = [&](int s) { return b0 + 8u * (10 + s); };
  auto p_ready = [&](int s) { return b0 + 8u * (12 + s); };
  auto s_free = [&](int s) { return b0 + 8u * (14 + s); };
  const uint32_t o_done = b0 + 8u * 16;
  auto o_final = [&](int s) { return b0 + 8u * (17 + s); };
  auto o_empty = [&](int s) { return b0 + 8u * (19 + s); };
  const uint32_t drain = b0 + 8u * 21;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.G, TQ = TQ_ROWS / G;
  const int items = a.qtiles * a.nkv * a.num_seqs;

  // Item i -> (sequence, KV head, query tile) and its extent; false when the tile is empty.
  struct Item {
    int b, h, qs, q_len, t0, k_len, off, n_tiles;
  };
  auto item = [&](int i, Item& it) -> bool {
    const int per = a.nkv * a.num_seqs;
    const int qt = a.qtiles - 1 - i / per;
    const int rem = i % per;
    it.h = rem / a.num_seqs;
    it.b = rem % a.num_seqs + a.seq_offset;
    it.qs = a.cu_q[it.b];
    it.q_len = a.cu_q[it.b + 1] - it.qs;
    it.t0 = qt * TQ;
    if (it.t0 >= it.q_len) return false;
    it.k_len = a.ctx_lens[it.b];
    it.off = it.k_len - it.q_len;
    const int kmax = min(it.k_len, it.off + min(it.q_len, it.t0 + TQ));
    it.n_tiles = (kmax + TK - 1) / TK;
    return it.n_tiles > 0;
  };

  if (threadIdx.x == 0) {
    bar_init(q_full, 1);
    bar_init(q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      bar_init(k_full(s), 1);
      bar_init(k_empty(s), 1);
      bar_init(v_full(s), 1);
      bar_init(v_empty(s), 1);
      bar_init(s_full(s), 1);
      bar_init(p_ready(s), 256);
      bar_init(s_free(s), 1);
      bar_init(o_final(s), 1);
      bar_init(o_empty(s), 256);
    }
    bar_init(o_done, 1);
    bar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)), "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tslot;

  auto wait = [&](uint32_t bar, uint32_t parity, int code) -> bool {
    if (att_try(bar, parity)) return true;
    SpinBudget sb;
    while (!att_try(bar, parity)) {
      if (*abort_flag) return false;
      if (sb.expired(ATT_WAIT_NS)) {
        atomicCAS(&g_attn_error, 0, code);
        *abort_flag = 1;
        return false;
      }
    }
    return true;
  };
  // Exit path: waits for a phase regardless of the abort flag (bounded), so no copy or MMA
  // of this CTA is still writing shared memory or TMEM when the CTA frees them.
  auto settle = [&](uint32_t bar, uint32_t parity) {
    SpinBudget sb;
    while (!att_try(bar, parity))
      if (sb.expired(ATT_WAIT_NS)) {
        atomicCAS(&g_attn_error, 0, 51);
        return;
      }
  };

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------------ TMA producer
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&qmap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&kmap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&vmap)) : "memory");
    const int boxes = TK / a.kv_box;
    bool ok = true;
    int g = 0, n_it = 0;
    int last[2][2] = {{-1, -1}, {-1, -1}};  // [K/V][stage]: tile of the last load issued there
    for (int i = blockIdx.x; i < items && ok; i += gridDim.x) {
      Item it;
      if (!item(i, it)) continue;
      // the previous item's S MMAs are done reading Q
      if (n_it >= 1 && !wait(q_empty, (n_it - 1) & 1, 49)) break;
      ++n_it;
      expect_tx(q_full, TILE);
      for (int half = 0; half < 2; ++half)
        tma3d(smem_u32(sq + half * HALF), &qmap, q_full, half * 64, it.h * G, it.qs + it.t0);
      const int* bt = a.block_tables + (int64_t)it.b * a.W;
      for (int j = 0; j < it.n_tiles && ok; ++j, ++g) {
        const int s = g & 1;
        const uint32_t par = ((g >> 1) & 1) ^ 1;
        for (int kv = 0; kv < 2 && ok; ++kv) {
          if (!wait(kv ? v_empty(s) : k_empty(s), par, 40)) {
            ok = false;
            break;
          }
          const uint32_t full = kv ? v_full(s) : k_full(s);
          uint8_t* dst = (kv ? sv : sk) + s * TILE;
          last[kv][s] = g;
          expect_tx(full, TILE);
          for (int bx = 0; bx < boxes; ++bx) {
            const int tk = j * TK + bx * a.kv_box;
            const int bi = tk / a.block_size;
            int row = a.kv_rows;  // past the end: the box reads as zeros
            if (tk < it.k_len && bi < a.W) {
              const int blk = bt[bi];
              if (blk >= 0 && blk < a.num_blocks) row = (blk * a.nkv + it.h) * a.block_size + (tk % a.block_size);
            }
            for (int half = 0; half < 2; ++half)
              tma2d(smem_u32(dst + half * HALF + bx * a.kv_box * 128), kv ? &vmap : &kmap, full, half * 64, row);
          }
        }
      }
    }
    if (*abort_flag) {  // loads nobody consumed may still be landing
      if (n_it) settle(q_full, (n_it - 1) & 1);
      for (int kv = 0; kv < 2; ++kv)
        for (int s = 0; s < 2; ++s)
          if (last[kv][s] >= 0) settle(kv ? v_full(s) : k_full(s), (last[kv][s] >> 1) & 1);
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------------ MMA issuer
    const uint32_t id_qk = idesc(false), id_pv = idesc(true);
    const uint32_t qa = smem_u32(sq);
    bool ok = true;
    int g = 0, n_it = 0;
    for (int i = blockIdx.x; i < items && ok; i += gridDim.x) {
      Item it;
      if (!item(i, it)) continue;
      const int ob = n_it & 1;
      if (!wait(q_full, n_it & 1, 41)) break;
      const int n = it.n_tiles;
      for (int j = 0; j <= n && ok; ++j) {
        if (j < n) {
          const int gs = g + j, s = gs & 1;
          if (!wait(k_full(s), (gs >> 1) & 1, 42)) { ok = false; break; }
          // no tcgen05 fence here: both waits are on TMA or tcgen05.commit arrivals, which order the
          // data this MMA reads and the TMEM it overwrites (the fence is needed after p_ready, below)
          if (gs >= 2 && !wait(s_free(s), ((gs - 2) >> 1) & 1, 43)) { ok = false; break; }
          const uint32_t kb = smem_u32(sk + s * TILE);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t ho = (k >> 2) * HALF + (k & 3) * 32;  // 16-element step inside a 64-dim half
            mma_ss(tmem + s_col(s), desc_sw128(qa + ho, 16, 1024), desc_sw128(kb + ho, 16, 1024), id_qk, k > 0);
          }
          commit(s_full(s));
          commit(k_empty(s));
          if (j == n - 1) commit(q_empty);  // every S MMA of this item reads Q before this completes
        }
        if (j >= 1) {
          const int gp = g + j - 1, s = gp & 1;
          if (!wait(p_ready(s), (gp >> 1) & 1, 44)) { ok = false; break; }
          if (!wait(v_full(s), (gp >> 1) & 1, 45)) { ok = false; break; }
          // O[ob] was last used by the item two before this one: its output must have been read
          if (j == 1 && n_it >= 2 && !wait(o_empty(ob), ((n_it >> 1) - 1) & 1, 50)) { ok = false; break; }
          fence_after();
          const uint32_t vb = smem_u32(sv + s * TILE);
#pragma unroll
          for (int k = 0; k < 8; ++k)  // 16 keys per step: P columns 8k.., V rows 16k..
            mma_ts(tmem + o_col(ob), tmem + s_col(s) + 8 * k, desc_sw128(vb + k * 16 * 128, HALF, 1024), id_pv,
                   (j > 1 || k > 0) ? 1u : 0u);
          commit(o_done);
          commit(v_empty(s));
          commit(s_free(s));
        }
      }
      if (!ok) break;
      commit(o_final(ob));
      g += n;
      ++n_it;
    }
    commit(drain);  // completes when every MMA this thread issued has completed
    settle(drain, 0);
  } else if (warp >= 2) {
    // ------------------------------------------------------------------ softmax / output
    // Two warps per TMEM lane quarter: warp w serves rows 32 (w & 3) .. +31 and the key (and
    // head-dim) half `half` of them; the pair exchanges its row maxima through shared memory
    // (named barrier 1 + quarter, 64 threads) so both halves scale by the same maximum.
    const int q4 = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = q4 * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q4 * 32) << 16);
    const int c0 = half * 64;  // this thread's first key column of a tile / first head dim
    __shared__ float xmax[2][2][TQ_ROWS];  // [tile parity][half][row]
    __shared__ int xok[2][2][TQ_ROWS];
    __shared__ float xsum[2][TQ_ROWS];
    __shared__ int xokf[2][TQ_ROWS];
    // Both warps of a pair pass the same sequence of pair barriers on every path (errors
    // included): both walk every item, and each decision to stop a tile loop is taken from the
    // exchanged flags, identically by both.  After an error the remaining items cost one
    // exchange each and touch no barrier, TMEM or output.
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(1 + q4) : "memory"); };
    bool ok = true;
    int g = 0, n_it = 0;
    for (int i = blockIdx.x; i < items; i += gridDim.x) {
      Item it;
      if (!item(i, it)) continue;
      const int ob = n_it & 1;
      const int t = it.t0 + r / G, gq = r % G;
      const int pos = it.off + t;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < it.n_tiles; ++j) {
        const int gs = g + j, s = gs & 1;
        if (ok) ok = wait(s_full(s), (gs >> 1) & 1, 46);
        fence_after();
        uint32_t raw[64];
        if (ok) {
          tmem_ld32(lane_base + s_col(s) + c0, raw);
          tmem_ld32(lane_base + s_col(s) + c0 + 32, raw + 32);
          tmem_ld_wait();
        }
        const int lim = ok ? min(pos + 1, it.k_len) - j * TK - c0 : 0;  // keys [0, lim) of this half are visible
        float x[64];
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          x[c] = c < lim ? __uint_as_float(raw[c]) * a.scale_log2 : -INFINITY;
          mx = fmaxf(mx, x[c]);
        }
        xmax[s][half][r] = mx;
        xok[s][half][r] = ok ? 1 : 0;
        pair_sync();
        mx = fmaxf(xmax[s][0][r], xmax[s][1][r]);
        ok = xok[s][0][r] && xok[s][1][r];
        if (!ok) break;  // identical in both warps of the pair
        if (mx > m_used + RESCALE_LOG2 || m_used == -INFINITY) {
          // raise the running maximum; O (if any) must be rescaled first (each half its 64 dims)
          const float m_new = mx;
          if (j > 0 && m_used != -INFINITY) {
            if (!wait(o_done, (gs - 1) & 1, 47)) {
              ok = false;  // reported to the partner at the next exchange
            } else {
              fence_after();
              const float f = exp2f(m_used - m_new);
#pragma unroll 1
              for (int c = 0; c < 64; c += 32) {
                uint32_t o[32];
                tmem_ld32(lane_base + o_col(ob) + c0 + c, o);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
                tmem_st32(lane_base + o_col(ob) + c0 + c, o);
              }
              tmem_st_wait();
              l *= f;
            }
          }
          if (m_new != -INFINITY) m_used = m_new;
        }
        const float base = m_used == -INFINITY ? 0.f : m_used;
        uint32_t pk[32];
        float rs = 0.f;
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          const float p0 = exp2f(x[c] - base), p1 = exp2f(x[c + 1] - base);
          rs += p0 + p1;
          pk[c / 2] = pack_bf16(p0, p1);
        }
        l += rs;
        tmem_st32(lane_base + s_col(s) + half * 32, pk);  // keys c0.. -> packed columns 32 half ..
        tmem_st_wait();
        fence_before();
        arrive(p_ready(s));
      }
      // row sum over both halves (both warps of the pair reach this barrier on every path)
      xsum[half][r] = l;
      xokf[half][r] = ok ? 1 : 0;
      pair_sync();
      const float lt = xsum[0][r] + xsum[1][r];
      ok = xokf[0][r] && xokf[1][r];
      pair_sync();  // xsum / xok are rewritten by the next item
      if (ok && wait(o_final(ob), (n_it >> 1) & 1, 48)) {
        fence_after();
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
        __nv_bfloat16* dst = a.out + ((int64_t)(it.qs + t) * a.nq + it.h * G + gq) * 128 + c0;
        const bool valid = t < it.q_len;
#pragma unroll 1
        for (int c = 0; c < 64; c += 32) {
          uint32_t o[32];
          tmem_ld32(lane_base + o_col(ob) + c0 + c, o);
          tmem_ld_wait();
          if (valid) {
            float f[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(o[e]) * inv;
#pragma unroll
            for (int e = 0; e < 32; e += 8) *reinterpret_cast<uint4*>(dst + c + e) = f32_to_bf16x8(f + e);
          }
        }
        fence_before();
        arrive(o_empty(ob));
      } else {
        ok = false;
      }
      g += it.n_tiles;
      ++n_it;
    }
    fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

static int prefill_tc_smem() { return 1024 + pf::TILE * (1 + 2 * pf::NSTAGE) + 256; }

// 3-D view of q [T, nq, 128] for the packed (token, head) rows: box = 64 dims x G heads x 128/G tokens.
static bool q_map(CUtensorMap* m, const void* q, int T, int nq, int G) {
  auto enc = attn_encode();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)AD, (cuuint64_t)nq, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)AD * 2, (cuuint64_t)nq * AD * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)G, (cuuint32_t)(pf::TQ_ROWS / G)};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D view [num_blocks * nkv * block_size rows, 128 dims] of a bf16 K or V pool, box 64 x box_rows.
static bool kv_map_tc(CUtensorMap* m, const void* base, int64_t rows, int box_rows) {
  auto enc = attn_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)AD, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)AD * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Whether the tcgen05 prefill kernel serves this launch (bf16 KV, GQA group dividing 128).
static bool prefill_tc_ok(const AttnLaunch& L) {
  const int G = L.nq / L.nkv;
  if (L.kv_fp8 || L.head_dim != AD || L.nq % L.nkv || G < 1 || 128 % G) return false;
  if (L.block_size < 8) return false;  // a K/V box holds at least 8 rows (one swizzle group)
  if (((uintptr_t)L.q & 15) || ((uintptr_t)L.k_cache & 15) || ((uintptr_t)L.v_cache & 15)) return false;
  const int64_t rows = (int64_t)L.num_blocks * L.nkv * L.block_size;
  return rows < (int64_t)INT32_MAX - 256;
}

static cudaError_t launch_attn_prefill_tc(const AttnLaunch& L, int max_q_len, int total_q, cudaStream_t stream) {
  const int G = L.nq / L.nkv;
  pf::Args a;
  a.block_tables = L.block_tables;
  a.W = L.W;
  a.cu_q = L.cu_q;
  a.ctx_lens = L.ctx_lens;
  a.out = static_cast<__nv_bfloat16*>(L.out);
  a.nq = L.nq;
  a.nkv = L.nkv;
  a.G = G;
  a.block_size = L.block_size;
  a.num_blocks = L.num_blocks;
  a.seq_offset = L.seq_offset;
  a.kv_box = L.block_size < pf::TK ? L.block_size : pf::TK;
  const int64_t rows = (int64_t)L.num_blocks * L.nkv * L.block_size;
  a.kv_rows = (int)rows;
  a.scale_log2 = L.softmax_scale * LOG2E;
  CUtensorMap qm, km, vm;
  if (!q_map(&qm, L.q, total_q, L.nq, G) || !kv_map_tc(&km, L.k_cache, rows, a.kv_box) ||
      !kv_map_tc(&vm, L.v_cache, rows, a.kv_box))
    return cudaErrorInvalidValue;
  static std::atomic<uint64_t> done{0};
  cudaError_t e = smem_opt_in(done, attn_prefill_tc_kernel, prefill_tc_smem());
  if (e != cudaSuccess) return e;
  const int TQ = pf::TQ_ROWS / G;
  a.qtiles = (max_q_len + TQ - 1) / TQ;
  a.num_seqs = L.num_seqs;
  const int items = a.qtiles * L.nkv * L.num_seqs;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  dim3 grid(items < sms ? items : sms);  // persistent: one CTA per SM (shared memory and TMEM allow one)
  launch_pdl(attn_prefill_tc_kernel, grid, dim3(pf::THREADS), prefill_tc_smem(), stream, qm, km, vm, a);
  NVB_LAUNCH_CHECK();
  return cudaSuccess;
}

// 2-D view [num_blocks * nkv * block_size rows, 128 dims] of one layer's K or V pool.
static bool kv_map(CUtensorMap* m, const void* base, int64_t rows, bool fp8, int box_rows) {
  auto enc = attn_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)AD, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(fp8 ? AD : AD * 2)};
  cuuint32_t box[2] = {(cuuint32_t)(fp8 ? 128 : 64), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base),
             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int decode_fp8_smem(int G) {
  return 1024 + DSTAGES * 2 * KTILE * AD + 4 * G * AD * 4 + 4 * 16 * 2 * 4 + 2 * DSTAGES * 8 + 16;
}

static int decode_tma_smem(bool fp8, int G) {
  const int stage = 2 * (fp8 ? KTILE * AD : KTILE * ROWB);
  return 1024 + DSTAGES * stage + (fp8 ? 4 * 8192 : 0) + 4 * G * AD * 4 + 4 * 16 * 2 * 4 + 2 * DSTAGES * 8 + 16;
}

cudaError_t launch_attn_decode(const AttnLaunch& L, cudaStream_t stream) {
  if (L.num_seqs == 0) return cudaSuccess;
  if (L.head_dim != AD || L.nq % L.nkv || L.nq / L.nkv > 16) return cudaErrorInvalidValue;
  if (L.splits > 1 && (!L.part_o || !L.part_lse)) return cudaErrorInvalidValue;
  if (L.block_size & (L.block_size - 1)) return cudaErrorInvalidValue;
  if (((uintptr_t)L.k_cache & 15) || ((uintptr_t)L.v_cache & 15)) return cudaErrorMisalignedAddress;
  DecodeArgs da;
  AttnArgs& a = da.a;
  a.q = static_cast<const __nv_bfloat16*>(L.q);
  a.k_cache = L.k_cache;
  a.v_cache = L.v_cache;
  a.k_scale = L.k_scale;
  a.v_scale = L.v_scale;
  a.block_tables = L.block_tables;
  a.W = L.W;
  a.cu_q = L.cu_q;
  a.ctx_lens = L.ctx_lens;
  a.out = static_cast<__nv_bfloat16*>(L.out);
  a.part_o = L.part_o;
  a.part_lse = L.part_lse;
  a.nq = L.nq;
  a.nkv = L.nkv;
  a.block_size = L.block_size;
  a.num_blocks = L.num_blocks;
  a.splits = L.splits;
  a.seq_offset = L.seq_offset;
  a.scale_log2 = L.softmax_scale * LOG2E;
  da.rows_per_box = L.block_size < KTILE ? L.block_size : KTILE;
  da.kv_fp8 = L.kv_fp8;
  const int64_t rows = (int64_t)L.num_blocks * L.nkv * L.block_size;
  CUtensorMap km, vm;
  if (!kv_map(&km, L.k_cache, rows, L.kv_fp8, da.rows_per_box) || !kv_map(&vm, L.v_cache, rows, L.kv_fp8, da.rows_per_box))
    return cudaErrorInvalidValue;
  dim3 grid(L.splits, L.nkv, L.num_seqs);
  const int sm = decode_tma_smem(L.kv_fp8, L.nq / L.nkv);
  const int sm_max = decode_tma_smem(L.kv_fp8, 16);
  if (L.kv_fp8 && L.nq / L.nkv <= 8 && L.block_size >= 16) {
    static std::atomic<uint64_t> done{0};
    cudaError_t e = smem_opt_in(done, attn_decode_fp8_kernel, decode_fp8_smem(8));
    if (e != cudaSuccess) return e;
    launch_pdl(attn_decode_fp8_kernel, grid, dim3(160), decode_fp8_smem(L.nq / L.nkv), stream, km, vm, da);
  } else if (L.kv_fp8) {
    static std::atomic<uint64_t> done{0};
    cudaError_t e = smem_opt_in(done, attn_decode_tma_kernel<true>, sm_max);
    if (e != cudaSuccess) return e;
    launch_pdl(attn_decode_tma_kernel<true>, grid, dim3(160), sm, stream, km, vm, da);
  } else {
    static std::atomic<uint64_t> done{0};
    cudaError_t e = smem_opt_in(done, attn_decode_tma_kernel<false>, sm_max);
    if (e != cudaSuccess) return e;
    launch_pdl(attn_decode_tma_kernel<false>, grid, dim3(160), sm, stream, km, vm, da);
  }
  NVB_LAUNCH_CHECK();
  if (L.splits > 1) {
    launch_pdl(attn_combine_kernel, dim3(L.num_seqs * L.nq), dim3(AD), 0, stream, L.part_o, L.part_lse, L.cu_q, a.out, L.nq, L.splits,
                                                             L.seq_offset);
    NVB_LAUNCH_CHECK();
  }
  return cudaSuccess;
}

int attn_error_code(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_attn_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_attn_error, &z, sizeof(int));
  }
  return v;
}

cudaError_t launch_attn_prefill(const AttnLaunch& L, int max_q_len, cudaStream_t stream) {
  return launch_attn_prefill_ex(L, max_q_len, -1, 1, stream);
}

cudaError_t launch_attn_prefill_ex(const AttnLaunch& L, int max_q_len, int total_q, int use_tc, cudaStream_t stream) {
  if (L.num_seqs == 0 || max_q_len == 0) return cudaSuccess;
  if (L.head_dim != AD || L.nq % L.nkv) return cudaErrorInvalidValue;
  if (use_tc && total_q > 0 && prefill_tc_ok(L)) return launch_attn_prefill_tc(L, max_q_len, total_q, stream);
  AttnArgs a;
  a.q = static_cast<const __nv_bfloat16*>(L.q);
  a.k_cache = L.k_cache;
  a.v_cache = L.v_cache;
  a.k_scale = L.k_scale;
  a.v_scale = L.v_scale;
  a.block_tables = L.block_tables;
  a.W = L.W;
  a.cu_q = L.cu_q;
  a.ctx_lens = L.ctx_lens;
  a.out = static_cast<__nv_bfloat16*>(L.out);
  a.part_o = nullptr;
  a.part_lse = nullptr;
  a.nq = L.nq;
  a.nkv = L.nkv;
  a.block_size = L.block_size;
  a.num_blocks = L.num_blocks;
  a.splits = 1;
  a.seq_offset = L.seq_offset;
  a.scale_log2 = L.softmax_scale * LOG2E;
  dim3 grid((max_q_len + 63) / 64, L.num_seqs, L.nq);
  int sm = prefill_smem(L.kv_fp8);
  if (L.kv_fp8) {
    static std::atomic<uint64_t> done{0};
    cudaError_t e = smem_opt_in(done, attn_prefill_kernel<true>, sm);
    if (e != cudaSuccess) return e;
    launch_pdl(attn_prefill_kernel<true>, grid, dim3(128), sm, stream, a);
  } else {
    static std::atomic<uint64_t> done{0};
    cudaError_t e = smem_opt_in(done, attn_prefill_kernel<false>, sm);
    if (e != cudaSuccess) return e;
    launch_pdl(attn_prefill_kernel<false>, grid, dim3(128), sm, stream, a);
  }
  NVB_LAUNCH_CHECK();
  return cudaSuccess;
}

}  // namespace nvb
