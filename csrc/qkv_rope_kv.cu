// Fused per-head q/k RMSNorm + NeoX RoPE + paged KV-cache store, on the QKV GEMM output.
//
// Replaces, per layer, the reference's q_norm/k_norm (nanovllm/models/qwen3.py:100-101),
// the torch.compile'd RoPE (nanovllm/layers/RoPE.py:57-74) and the eager index_put KV
// store (nanovllm/layers/attention.py:139-189): one launch, one read of the QKV rows.
//
// Layouts: qkv [T, (nq + 2 nkv) * 128] bf16 (row stride qkv_stride); q_out [T, nq*128];
// caches [num_blocks, nkv, block_size, 128] (bf16 or fp8 e4m3); cos_sin [max_pos, 128]
// fp32 (first 64 cos, last 64 sin); slot = block * block_size + offset, -1 = skip.
//
// fp8 scales ([num_blocks, nkv] fp32 for K and for V): the step that writes offset 0 of
// a block sets that block-head's scale to absmax(first token) * 4 / 448; other tokens
// use it.  A token whose block's first token is written in the same launch recomputes
// that first token's values to derive the identical scale (no inter-CTA ordering).
#include <atomic>
#include "common.cuh"
#include "kernels.h"

namespace nvb {

constexpr int HD = 128;  // head_dim handled by this kernel (8 elements per lane, 16 lanes per head)

struct QkvPostArgs {
  const __nv_bfloat16* qkv;
  int64_t qkv_stride;
  __nv_bfloat16* q_out;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  float eps;
  const int* positions;
  const float* cos_sin;
  void* k_cache;
  void* v_cache;
  float* k_scale;
  float* v_scale;
  const int* slots;
  int T, nq, nkv, block_size;
  int kv_fp8;
  int num_blocks;  // pool blocks: slots must lie in [0, num_blocks * block_size) (-1: skip)
};

// Check word of this file: 402 a KV slot beyond the pool (access skipped), 403 a stage's bulk copy
// did not complete within the bound (the CTA stops).
__device__ int g_qkv_check = 0;

int qkv_check_code(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_qkv_check, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_qkv_check, &z, sizeof(int));
  }
  return v;
}

// Persistent, TMA-fed.  A chunk is R consecutive tokens: their QKV rows and the RoPE table rows of
// their positions are brought into a shared-memory stage by bulk copies (cp.async.bulk, completion
// counted by an mbarrier), STAGES chunks in flight per CTA, so the bytes in flight do not depend on
// registers (a register-fed version with 8 loads of 16 B in flight per lane reached 0.41 of the copy
// bandwidth).  Half a warp works on one head of one token: lane hl (0..15) holds elements
// [4 hl, 4 hl + 4) and [64 + 4 hl, 64 + 4 hl + 4), so both RoPE partners sit in the same lane; the
// head (and so every branch below) is uniform over the half.
constexpr int QKV_THREADS = 256;         // 16 half-warps
constexpr int QKV_STAGE_TARGET = 16384;  // bytes of QKV rows per stage (R = 1..16 tokens)
constexpr int QKV_SMEM_TARGET = 65536;   // stages per CTA: about this many bytes (3 CTAs per SM)
constexpr int QKV_MAX_SMEM = 200 * 1024;  // dynamic shared memory opt-in (static use is a few bytes)
constexpr uint64_t QKV_WAIT_NS = 2000000000ull;

__device__ __forceinline__ float half_sum(float v, unsigned hmask) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(hmask, v, o);
  return v;
}
__device__ __forceinline__ float half_max(float v, unsigned hmask) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(hmask, v, o));
  return v;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: two IEEE round-to-nearest operations per instruction,
// the same results as the scalar forms).
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mul.rn.f32x2 rd, ra, rb;\n"
      " mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rc, {%6, %7};\n"
      " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// RMSNorm with weights w (this lane's 8; nullptr: none), then NeoX rotation with the tables c / sn
// (cos / sin of frequencies 4 hl .. 4 hl + 3; nullptr: none) of the 8 elements x held by this lane
// (x[i] and x[4 + i] are elements 4 hl + i and 64 + 4 hl + i).  Explicit roundings (no contraction),
// so the scale of an fp8 block computed here and recomputed elsewhere in the launch agree bit for bit;
// pairs of elements go through the packed f32x2 forms (half the instructions, the same bits).
__device__ __forceinline__ void norm_rope(float eps, const float* w, const float* c, const float* sn,
                                          unsigned hmask, float* x) {
  // v[0..1]: elements 4 hl .. 4 hl + 3, v[2..3]: 64 + 4 hl .. (pairs of x)
  float2 v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = make_float2(x[2 * i], x[2 * i + 1]);
  if (w) {
    float2 acc = mul2(v[0], v[0]);
    acc = fma2(v[1], v[1], acc);
    acc = fma2(v[2], v[2], acc);
    acc = fma2(v[3], v[3], acc);
    float ss = __fadd_rn(acc.x, acc.y);
    ss = half_sum(ss, hmask);
    const float inv = rsqrtf(ss / (float)HD + eps);
    const float2 inv2 = make_float2(inv, inv);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = mul2(mul2(v[i], inv2), make_float2(w[2 * i], w[2 * i + 1]));
  }
  if (c) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float2 cc = make_float2(c[2 * i], c[2 * i + 1]), ss2 = make_float2(sn[2 * i], sn[2 * i + 1]);
      const float2 a = v[i], b = v[2 + i];
      const float2 bs = mul2(b, ss2);
      v[i] = fma2(a, cc, make_float2(-bs.x, -bs.y));  // a c - b s
      v[2 + i] = fma2(b, cc, mul2(a, ss2));           // b c + a s
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = v[i].x;
    x[2 * i + 1] = v[i].y;
  }
}

__device__ __forceinline__ void load_head(const __nv_bfloat16* head, int hl, float* x) {
  bf16x4_to_f32(*reinterpret_cast<const uint2*>(head + 4 * hl), x);
  bf16x4_to_f32(*reinterpret_cast<const uint2*>(head + 64 + 4 * hl), x + 4);
}
__device__ __forceinline__ void load_tables(const float* row, int hl, float* c, float* sn) {
  const float4 c0 = *reinterpret_cast<const float4*>(row + 4 * hl);
  const float4 s0 = *reinterpret_cast<const float4*>(row + 64 + 4 * hl);
  c[0] = c0.x; c[1] = c0.y; c[2] = c0.z; c[3] = c0.w;
  sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
}

__device__ __forceinline__ bool qkv_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for a stage (error 403 in the check word when it runs out).
__device__ __forceinline__ bool qkv_wait(uint32_t bar, uint32_t parity) {
  if (qkv_try(bar, parity)) return true;
  SpinBudget sb;
  while (!qkv_try(bar, parity)) {
    if (sb.expired(QKV_WAIT_NS)) {
      atomicCAS(&g_qkv_check, 0, 403);
      return false;
    }
  }
  return true;
}

// Warp 0 brings chunk c (tokens [c R, c R + Rc)) into the stage at `stage` with full barrier `bar`:
// lane i copies token i's QKV row and the RoPE table row of its position.
__device__ __forceinline__ void qkv_issue(const QkvPostArgs& a, int c, int R, int row_bytes, uint8_t* stage,
                                          uint32_t bar, int lane) {
  const int t0 = c * R;
  const int rc = min(R, a.T - t0);
  if (lane == 0)
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                 "r"((uint32_t)(rc * (row_bytes + HD * 4)))
                 : "memory");
  __syncwarp();
  for (int i = lane; i < rc; i += 32) {
    const int t = t0 + i;
    const void* src = a.qkv + (int64_t)t * a.qkv_stride;
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(stage + (size_t)i * row_bytes)),
        "l"(src), "r"((uint32_t)row_bytes), "r"(bar)
        : "memory");
    const float* tab = a.cos_sin + (int64_t)a.positions[t] * HD;
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(stage + (size_t)R * row_bytes + (size_t)i * HD * 4)),
        "l"(tab), "r"((uint32_t)(HD * 4)), "r"(bar)
        : "memory");
  }
}

// Per-token values shared by the token's K/V heads: the destination of head 0 in the paged cache
// (element offset; the next head is block_size * 128 further), and the block / offset of the slot.
struct KvDst {
  bool ok;  // slot >= 0 and inside the pool (a bad slot records 402 once and skips the token's K/V)
  int blk, off, first_t;
  bool first_here;  // fp8: the block's first token is written by this launch (derive its scale)
  int64_t base;
};

__device__ __forceinline__ KvDst kv_dst(const QkvPostArgs& a, int t, int hl) {
  KvDst d;
  const int slot = a.slots[t];
  d.ok = slot >= 0 && in_range(slot, (long long)a.num_blocks * a.block_size, &g_qkv_check, 402);
  d.blk = d.ok ? slot / a.block_size : 0;
  d.off = slot - d.blk * a.block_size;
  d.base = ((int64_t)d.blk * a.nkv * a.block_size + d.off) * HD + 4 * hl;
  d.first_t = t - d.off;
  d.first_here = d.ok && a.kv_fp8 && (d.off == 0 || (d.first_t >= 0 && a.slots[d.first_t] == slot - d.off));
  return d;
}

// Store head h of K (is_k) or V of one token into the paged cache: bf16, or e4m3 with the block's
// per-head scale.  x holds this lane's 8 elements, normed and rotated for K.
__device__ __forceinline__ void kv_store(const QkvPostArgs& a, const KvDst& d, bool is_k, int h, int j, int hl,
                                         unsigned hmask, const float* kw, const float* x) {
  const int64_t dst = d.base + (int64_t)h * a.block_size * HD;
  if (!a.kv_fp8) {
    __nv_bfloat16* cache = static_cast<__nv_bfloat16*>(is_k ? a.k_cache : a.v_cache);
    *reinterpret_cast<uint2*>(cache + dst) = f32_to_bf16x4(x);
    *reinterpret_cast<uint2*>(cache + dst + 64) = f32_to_bf16x4(x + 4);
    return;
  }
  float* scales = is_k ? a.k_scale : a.v_scale;
  float scale;
  if (d.first_here) {
    // this launch writes the block's first token: derive the scale from it (recomputed here when it
    // is another token, so every writer of the block agrees without ordering)
    float y[8];
    if (d.off == 0) {
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = x[e];
    } else {
      load_head(a.qkv + (int64_t)d.first_t * a.qkv_stride + j * HD, hl, y);
      if (is_k) {
        float c1[4], s1[4];
        load_tables(a.cos_sin + (int64_t)a.positions[d.first_t] * HD, hl, c1, s1);
        norm_rope(a.eps, kw, c1, s1, hmask, y);
      }
    }
    float m = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(y[e]));
    m = half_max(m, hmask);
    scale = fmaxf(m * (4.0f / 448.0f), 1e-8f);
    if (d.off == 0 && hl == 0) scales[(int64_t)d.blk * a.nkv + h] = scale;
  } else {
    scale = scales[(int64_t)d.blk * a.nkv + h];
  }
  const float inv = __frcp_rn(scale);  // 1 / scale, correctly rounded (the same bits as the division)
  float q0[4] = {x[0] * inv, x[1] * inv, x[2] * inv, x[3] * inv};
  float q1[4] = {x[4] * inv, x[5] * inv, x[6] * inv, x[7] * inv};
  uint8_t* cache = static_cast<uint8_t*>(is_k ? a.k_cache : a.v_cache);
  *reinterpret_cast<uint32_t*>(cache + dst) = f32x4_to_e4m3(q0);
  *reinterpret_cast<uint32_t*>(cache + dst + 64) = f32x4_to_e4m3(q1);
}

// Chunks c = blockIdx.x, + gridDim.x, ...; a ring of `stages` stages (each: R tokens' rows, then their
// R table rows, 16-byte aligned) with a full mbarrier (the copies' bytes) and an empty mbarrier (one
// arrival per warp done with the stage) each.  Warp 0 refills a stage once every warp has left it, so
// no warp waits for the others between chunks.  Half-warp w works on token w / P of the chunk
// (P = 16 / R half-warps per token) and heads w % P, + P, ...
__global__ void __launch_bounds__(QKV_THREADS, 3) qkv_post_kernel(QkvPostArgs a, int R, int stages) {
  extern __shared__ __align__(128) uint8_t qkv_smem[];
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, hl = lane & 15;
  const int hw = threadIdx.x >> 4;
  const unsigned hmask = 0xFFFFu << (16 * ((threadIdx.x >> 4) & 1));
  const int H = a.nq + 2 * a.nkv;
  const int row_bytes = H * HD * 2;
  const int stage_bytes = R * (row_bytes + HD * 4);
  const int P = 16 / R;
  const int nchunks = (a.T + R - 1) / R;
  uint64_t* bars = reinterpret_cast<uint64_t*>(qkv_smem + (size_t)stages * stage_bytes);
  auto full = [&](int st) { return smem_u32(bars + st); };
  auto empty = [&](int st) { return smem_u32(bars + stages + st); };
  if (threadIdx.x == 0) {
    for (int st = 0; st < stages; ++st) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(full(st)));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(empty(st)), "r"(QKV_THREADS / 32));
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  int issued = 0;  // warp 0: chunks issued so far (iterations 0 .. issued - 1)
  if (warp == 0)
    for (int st = 0; st < stages; ++st) {
      const int c = blockIdx.x + st * gridDim.x;
      if (c >= nchunks) break;
      qkv_issue(a, c, R, row_bytes, qkv_smem + (size_t)st * stage_bytes, full(st), lane);
      ++issued;
    }
  float qw[8], kw[8];
  bf16x4_to_f32(*reinterpret_cast<const uint2*>(a.q_norm + 4 * hl), qw);
  bf16x4_to_f32(*reinterpret_cast<const uint2*>(a.q_norm + 64 + 4 * hl), qw + 4);
  bf16x4_to_f32(*reinterpret_cast<const uint2*>(a.k_norm + 4 * hl), kw);
  bf16x4_to_f32(*reinterpret_cast<const uint2*>(a.k_norm + 64 + 4 * hl), kw + 4);
  const int tok = hw / P, hp = hw - tok * P;
  int it = 0;
  bool failed = false;
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x, ++it) {
    const int s = it % stages;
    const uint32_t ph = (uint32_t)(it / stages) & 1u;
    if (!__all_sync(FULL_MASK, qkv_wait(full(s), ph))) {  // warp-uniform: the warp leaves together
      failed = true;
      break;
    }
    const uint8_t* stage = qkv_smem + (size_t)s * stage_bytes;
    if (c * R + tok < a.T) {
      // heads hp, hp + P, ... of token t: first its query heads, then key heads, then value heads
      const int t = c * R + tok;
      const __nv_bfloat16* row = reinterpret_cast<const __nv_bfloat16*>(stage + (size_t)tok * row_bytes);
      float cs[4], sn[4];
      load_tables(reinterpret_cast<const float*>(stage + (size_t)R * row_bytes + (size_t)tok * HD * 4), hl, cs, sn);
      int j = hp;
      __nv_bfloat16* qdst = a.q_out + (int64_t)t * a.nq * HD + 4 * hl;
      for (; j < a.nq; j += P) {
        float x[8];
        load_head(row + j * HD, hl, x);
        norm_rope(a.eps, qw, cs, sn, hmask, x);
        *reinterpret_cast<uint2*>(qdst + j * HD) = f32_to_bf16x4(x);
        *reinterpret_cast<uint2*>(qdst + j * HD + 64) = f32_to_bf16x4(x + 4);
      }
      if (j < H) {
        const KvDst d = kv_dst(a, t, hl);
        for (; j < a.nq + a.nkv; j += P) {
          float x[8];
          load_head(row + j * HD, hl, x);
          norm_rope(a.eps, kw, cs, sn, hmask, x);
          if (d.ok) kv_store(a, d, true, j - a.nq, j, hl, hmask, kw, x);
        }
        for (; j < H; j += P) {
          float x[8];
          load_head(row + j * HD, hl, x);
          if (d.ok) kv_store(a, d, false, j - a.nq - a.nkv, j, hl, hmask, kw, x);
        }
      }
    }
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(empty(s)) : "memory");
    const int cn = c + stages * gridDim.x;
    if (warp == 0 && cn < nchunks) {
      int ok = 1;
      if (lane == 0) ok = qkv_wait(empty(s), ph);  // every warp has left stage s
      if (!__shfl_sync(FULL_MASK, ok, 0)) {
        failed = true;
        break;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic reads before the async refill
      qkv_issue(a, cn, R, row_bytes, qkv_smem + (size_t)s * stage_bytes, full(s), lane);
      ++issued;
    }
  }
  if (failed && threadIdx.x == 0) {
    // a wait ran out: let the copies already issued land before the CTA's shared memory goes away
    // (each wait bounded; the first that also runs out ends the drain)
    for (int i = it; i < issued; ++i)
      if (!qkv_wait(full(i % stages), (uint32_t)(i / stages) & 1u)) break;
  }
}

// Chunk size R (tokens per stage) and stage count for rows of H heads.
static void qkv_plan(int H, int* R, int* stages) {
  const int row_bytes = H * HD * 2;
  int r = 1;
  while (r < 16 && 2 * r * row_bytes <= QKV_STAGE_TARGET) r *= 2;
  const int stage = r * (row_bytes + HD * 4);
  int s = QKV_SMEM_TARGET / stage;
  *R = r;
  *stages = s < 2 ? 2 : (s > 6 ? 6 : s);
}

cudaError_t launch_qkv_post(const void* qkv, int64_t qkv_stride, void* q_out, const void* q_norm, const void* k_norm,
                            float eps, const int* positions, const float* cos_sin, void* k_cache, void* v_cache,
                            float* k_scale, float* v_scale, const int* slots, int T, int nq, int nkv, int head_dim,
                            int block_size, int kv_fp8, cudaStream_t stream, int num_blocks) {
  if (T == 0) return cudaSuccess;
  if (head_dim != HD || nq <= 0 || nkv <= 0 || block_size <= 0) return cudaErrorInvalidValue;
  // bulk copies and 8-byte accesses: rows, norm weights, RoPE tables and caches start on 16-byte boundaries
  auto al16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  if (qkv_stride % 8 || !al16(qkv) || !al16(q_out) || !al16(q_norm) || !al16(k_norm) || !al16(cos_sin) ||
      !al16(k_cache) || !al16(v_cache))
    return cudaErrorInvalidValue;
  QkvPostArgs a;
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.qkv_stride = qkv_stride;
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.q_norm = static_cast<const __nv_bfloat16*>(q_norm);
  a.k_norm = static_cast<const __nv_bfloat16*>(k_norm);
  a.eps = eps;
  a.positions = positions;
  a.cos_sin = cos_sin;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.slots = slots;
  a.T = T;
  a.nq = nq;
  a.nkv = nkv;
  a.block_size = block_size;
  a.kv_fp8 = kv_fp8;
  a.num_blocks = num_blocks;
  const int H = nq + 2 * nkv;
  int R, stages;
  qkv_plan(H, &R, &stages);
  const int smem = stages * R * (H * HD * 2 + HD * 4) + stages * 16;
  if (smem > QKV_MAX_SMEM) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_done{0};  // one opt-in (the largest size) per device
  cudaError_t e = smem_opt_in(attr_done, qkv_post_kernel, QKV_MAX_SMEM);
  if (e != cudaSuccess) return e;
  // resident CTAs per SM (registers and shared memory), once per device and stage size: the grid
  // is one wave, every CTA loops over its chunks
  // one word per device, (smem << 32) | (SMs << 16) | CTAs per SM, so a reader never sees a
  // mix of two entries
  static std::atomic<uint64_t> occ[64];
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = 0, per_sm = 0;
  const uint64_t w = dev >= 0 && dev < 64 ? occ[dev].load(std::memory_order_relaxed) : 0;
  if (w && (int)(w >> 32) == smem) {
    sms = (int)((w >> 16) & 0xffff);
    per_sm = (int)(w & 0xffff);
  } else {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qkv_post_kernel, QKV_THREADS, (size_t)smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64 && sms > 0 && sms < 65536 && per_sm > 0 && per_sm < 65536)
      occ[dev].store(((uint64_t)smem << 32) | ((uint64_t)sms << 16) | (uint64_t)per_sm, std::memory_order_relaxed);
  }
  if (sms <= 0) sms = 148;
  if (per_sm <= 0) per_sm = 1;
  const int64_t nchunks = ((int64_t)T + R - 1) / R;
  const int64_t grid = nchunks < (int64_t)sms * per_sm ? nchunks : (int64_t)sms * per_sm;
  launch_pdl(qkv_post_kernel, dim3((unsigned)grid), dim3(QKV_THREADS), (size_t)smem, stream, a, R, stages);
  NVB_LAUNCH_CHECK();
  return cudaSuccess;
}

}  // namespace nvb
