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

__device__ int g_qkv_check = 0;  // bounds-check word of this file (402: KV slot beyond the pool)

int qkv_check_code(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_qkv_check, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_qkv_check, &z, sizeof(int));
  }
  return v;
}

// Half a warp per head: lane hl (0..15) of the half holds elements [8 hl, 8 hl + 8) of the
// head's 128, so every access is 16 bytes and the RoPE partner of element e (e +- 64) sits in
// lane hl ^ 8 of the same half.  `hmask` names the 16 lanes of the half; the head (and so every
// branch below) is uniform over them.
constexpr int QKV_HPW = 16;  // heads per warp (two per pass, one per half); 8 loads in flight per lane

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

// RoPE tables of one position for this lane's 8 elements (cos, sin of frequencies (8 hl) & 63 ..).
__device__ __forceinline__ void rope_tables(const float* cos_sin, int pos, int hl, float* c, float* sn) {
  const float* cs = cos_sin + (int64_t)pos * HD + ((hl * 8) & 63);
  const float4 c0 = *reinterpret_cast<const float4*>(cs), c1 = *reinterpret_cast<const float4*>(cs + 4);
  const float4 s0 = *reinterpret_cast<const float4*>(cs + 64), s1 = *reinterpret_cast<const float4*>(cs + 68);
  c[0] = c0.x; c[1] = c0.y; c[2] = c0.z; c[3] = c0.w; c[4] = c1.x; c[5] = c1.y; c[6] = c1.z; c[7] = c1.w;
  sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w; sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
}

// RMSNorm with the head's weights nw (nullptr: none; this lane reads its 8), then NeoX rotation
// with tables c / sn (nullptr: none) of the 8 elements x of one head held by this lane.
__device__ __forceinline__ void norm_rope8(float eps, const __nv_bfloat16* nw, const float* c, const float* sn,
                                           int hl, unsigned hmask, float* x) {
  if (nw) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
    ss = half_sum(ss, hmask);
    const float inv = rsqrtf(ss / (float)HD + eps);
    float w[8];
    bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(nw + hl * 8)), w);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = x[i] * inv * w[i];
  }
  if (c) {
    float p[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = __shfl_xor_sync(hmask, x[i], 8);
    const float sign = hl < 8 ? -1.f : 1.f;  // first half: x c - x[e + 64] s; second: x c + x[e - 64] s
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = x[i] * c[i] + sign * p[i] * sn[i];
  }
}

// One warp per (token, group of QKV_HPW heads); all of the group's rows are requested before the
// first is processed (a warp per head with one 8-byte load per lane in flight was latency-bound
// at a third of the copy bandwidth).
__global__ void __launch_bounds__(128, 4) qkv_post_kernel(QkvPostArgs a) {
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  const int lane = threadIdx.x & 31, hl = lane & 15, half = lane >> 4;
  const unsigned hmask = 0xFFFFu << (16 * half);
  const int heads = a.nq + 2 * a.nkv;
  const int groups = (heads + QKV_HPW - 1) / QKV_HPW;
  const int64_t gw = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (gw >= (int64_t)a.T * groups) return;
  const int t = (int)(gw / groups);
  const int j0 = (int)(gw - (int64_t)t * groups) * QKV_HPW;
  const __nv_bfloat16* row = a.qkv + (int64_t)t * a.qkv_stride + hl * 8;
  uint4 raw[QKV_HPW / 2];
#pragma unroll
  for (int i = 0; i < QKV_HPW / 2; ++i) {
    const int j = j0 + 2 * i + half;
    if (j < heads) raw[i] = *reinterpret_cast<const uint4*>(row + j * HD);
  }
  float c[8], sn[8];
  const bool any_rope = j0 < a.nq + a.nkv;
  if (any_rope) rope_tables(a.cos_sin, a.positions[t], hl, c, sn);
  const int slot = j0 + QKV_HPW > a.nq ? a.slots[t] : -1;
#pragma unroll
  for (int i = 0; i < QKV_HPW / 2; ++i) {
    const int j = j0 + 2 * i + half;
    if (j >= heads) continue;  // uniform over the half
    float x[8];
    bf16x8_to_f32(raw[i], x);
    if (j < a.nq) {
      norm_rope8(a.eps, a.q_norm, c, sn, hl, hmask, x);
      *reinterpret_cast<uint4*>(a.q_out + (int64_t)t * a.nq * HD + j * HD + hl * 8) = f32_to_bf16x8(x);
      continue;
    }
    const bool is_k = j < a.nq + a.nkv;
    const int h = is_k ? j - a.nq : j - a.nq - a.nkv;
    norm_rope8(a.eps, is_k ? a.k_norm : nullptr, is_k ? c : nullptr, sn, hl, hmask, x);
    if (slot < 0) continue;
    if (!in_range(slot, (long long)a.num_blocks * a.block_size, &g_qkv_check, 402)) continue;
    const int blk = slot / a.block_size, off = slot - blk * a.block_size;
    const int64_t dst = (((int64_t)blk * a.nkv + h) * a.block_size + off) * HD + hl * 8;
    if (!a.kv_fp8) {
      __nv_bfloat16* cache = static_cast<__nv_bfloat16*>(is_k ? a.k_cache : a.v_cache);
      *reinterpret_cast<uint4*>(cache + dst) = f32_to_bf16x8(x);
      continue;
    }
    float* scales = is_k ? a.k_scale : a.v_scale;
    float scale;
    const int first_t = t - off;
    if (off == 0 || (first_t >= 0 && a.slots[first_t] == slot - off)) {
      // this launch writes the block's first token: derive the scale from it (recomputed here
      // when it is another token, so every writer of the block agrees without ordering)
      float y[8];
      if (off == 0) {
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = x[e];
      } else {
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.qkv + (int64_t)first_t * a.qkv_stride + j * HD + hl * 8), y);
        if (is_k) {
          float c1[8], s1[8];
          rope_tables(a.cos_sin, a.positions[first_t], hl, c1, s1);
          norm_rope8(a.eps, a.k_norm, c1, s1, hl, hmask, y);
        }
      }
      float m = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(y[e]));
      m = half_max(m, hmask);
      scale = fmaxf(m * (4.0f / 448.0f), 1e-8f);
      if (off == 0 && hl == 0) scales[(int64_t)blk * a.nkv + h] = scale;
    } else {
      scale = scales[(int64_t)blk * a.nkv + h];
    }
    const float inv = 1.0f / scale;
    float q0[4] = {x[0] * inv, x[1] * inv, x[2] * inv, x[3] * inv};
    float q1[4] = {x[4] * inv, x[5] * inv, x[6] * inv, x[7] * inv};
    uint8_t* cache = static_cast<uint8_t*>(is_k ? a.k_cache : a.v_cache);
    *reinterpret_cast<uint2*>(cache + dst) = make_uint2(f32x4_to_e4m3(q0), f32x4_to_e4m3(q1));
  }
}

cudaError_t launch_qkv_post(const void* qkv, int64_t qkv_stride, void* q_out, const void* q_norm, const void* k_norm,
                            float eps, const int* positions, const float* cos_sin, void* k_cache, void* v_cache,
                            float* k_scale, float* v_scale, const int* slots, int T, int nq, int nkv, int head_dim,
                            int block_size, int kv_fp8, cudaStream_t stream, int num_blocks) {
  if (T == 0) return cudaSuccess;
  if (head_dim != HD) return cudaErrorInvalidValue;
  // 16-byte accesses: rows, norm weights, RoPE tables and caches start on 16-byte boundaries
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
  int64_t warps = (int64_t)T * ((nq + 2 * nkv + QKV_HPW - 1) / QKV_HPW);
  int64_t blocks = (warps + 3) / 4;
  launch_pdl(qkv_post_kernel, dim3((unsigned)blocks), dim3(128), 0, stream, a);
  NVB_LAUNCH_CHECK();
  return cudaSuccess;
}

}  // namespace nvb
