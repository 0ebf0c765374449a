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

constexpr int HD = 128;  // head_dim handled by this kernel (4 elements per lane)

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

// Load 4 lanes' worth (4 elements) of head `head` of token t, optionally normalise with
// `nw` and rotate at `pos`.  Every lane of the warp must call it (uses shuffles).
__device__ __forceinline__ void load_head(const QkvPostArgs& a, int t, int head, const __nv_bfloat16* nw, bool rope,
                                          int lane, float* x) {
  const __nv_bfloat16* src = a.qkv + (int64_t)t * a.qkv_stride + head * HD + lane * 4;
  bf16x4_to_f32(*reinterpret_cast<const uint2*>(src), x);
  if (nw) {
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    ss = warp_sum(ss);
    float inv = rsqrtf(ss / (float)HD + a.eps);
    float w[4];
    bf16x4_to_f32(*reinterpret_cast<const uint2*>(nw + lane * 4), w);
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = x[i] * inv * w[i];
  }
  if (rope) {
    const int pos = a.positions[t];
    const float* cs = a.cos_sin + (int64_t)pos * HD;
    const int f = (lane * 4) & 63;
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(FULL_MASK, x[i], 16);
    const bool lo = lane < 16;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float c = cs[f + i], s = cs[64 + f + i];
      x[i] = lo ? (x[i] * c - p[i] * s) : (x[i] * c + p[i] * s);
    }
  }
}

constexpr int QKV_HPW = 8;  // heads per warp: their loads are all issued before any is used

// Normalise (nw) and rotate (at pos) the 4 elements x of one head held by this lane.
__device__ __forceinline__ void norm_rope(const QkvPostArgs& a, const __nv_bfloat16* nw, bool rope, const float* cs,
                                          int lane, float* x) {
  if (nw) {
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)HD + a.eps);
    float w[4];
    bf16x4_to_f32(*reinterpret_cast<const uint2*>(nw + lane * 4), w);
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = x[i] * inv * w[i];
  }
  if (rope) {
    const int f = (lane * 4) & 63;
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(FULL_MASK, x[i], 16);
    const bool lo = lane < 16;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float c = cs[f + i], sn = cs[64 + f + i];
      x[i] = lo ? (x[i] * c - p[i] * sn) : (x[i] * c + p[i] * sn);
    }
  }
}

// One warp per (token, group of QKV_HPW heads): every head's 256-byte row is requested before
// the first one is processed, so each warp keeps QKV_HPW loads in flight (one load per warp
// left the kernel latency-bound at a third of the copy bandwidth).
__global__ void __launch_bounds__(128) qkv_post_kernel(QkvPostArgs a) {
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  const int lane = threadIdx.x & 31;
  const int heads = a.nq + 2 * a.nkv;
  const int groups = (heads + QKV_HPW - 1) / QKV_HPW;
  const int64_t gw = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (gw >= (int64_t)a.T * groups) return;
  const int t = (int)(gw / groups);
  const int j0 = (int)(gw - (int64_t)t * groups) * QKV_HPW;
  const __nv_bfloat16* row = a.qkv + (int64_t)t * a.qkv_stride + lane * 4;
  uint2 raw[QKV_HPW];
#pragma unroll
  for (int i = 0; i < QKV_HPW; ++i)
    if (j0 + i < heads) raw[i] = *reinterpret_cast<const uint2*>(row + (j0 + i) * HD);
  const bool any_rope = j0 < a.nq + a.nkv;
  const float* cs = any_rope ? a.cos_sin + (int64_t)a.positions[t] * HD : nullptr;
  const int slot = j0 + QKV_HPW > a.nq ? a.slots[t] : -1;
#pragma unroll
  for (int i = 0; i < QKV_HPW; ++i) {
    const int j = j0 + i;
    if (j >= heads) break;
    float x[4];
    bf16x4_to_f32(raw[i], x);
    if (j < a.nq) {
      norm_rope(a, a.q_norm, true, cs, lane, x);
      *reinterpret_cast<uint2*>(a.q_out + (int64_t)t * a.nq * HD + j * HD + lane * 4) = f32_to_bf16x4(x);
      continue;
    }
    const bool is_k = j < a.nq + a.nkv;
    const int h = is_k ? j - a.nq : j - a.nq - a.nkv;
    const __nv_bfloat16* nw = is_k ? a.k_norm : nullptr;
    norm_rope(a, nw, is_k, cs, lane, x);
    if (slot < 0) continue;
    if (!in_range(slot, (long long)a.num_blocks * a.block_size, &g_qkv_check, 402)) continue;
    const int blk = slot / a.block_size, off = slot - blk * a.block_size;
    const int64_t dst = (((int64_t)blk * a.nkv + h) * a.block_size + off) * HD + lane * 4;
    if (!a.kv_fp8) {
      __nv_bfloat16* cache = static_cast<__nv_bfloat16*>(is_k ? a.k_cache : a.v_cache);
      *reinterpret_cast<uint2*>(cache + dst) = f32_to_bf16x4(x);
      continue;
    }
    float* scales = is_k ? a.k_scale : a.v_scale;
    float scale;
    const int first_t = t - off;
    if (off == 0 || (first_t >= 0 && a.slots[first_t] == slot - off)) {
      float y[4];
      if (off == 0) {
        y[0] = x[0]; y[1] = x[1]; y[2] = x[2]; y[3] = x[3];
      } else {
        load_head(a, first_t, j, nw, is_k, lane, y);
      }
      float m = fmaxf(fmaxf(fabsf(y[0]), fabsf(y[1])), fmaxf(fabsf(y[2]), fabsf(y[3])));
      m = warp_max(m);
      scale = fmaxf(m * (4.0f / 448.0f), 1e-8f);
      if (off == 0 && lane == 0) scales[(int64_t)blk * a.nkv + h] = scale;
    } else {
      scale = scales[(int64_t)blk * a.nkv + h];
    }
    const float inv = 1.0f / scale;
    float q[4] = {x[0] * inv, x[1] * inv, x[2] * inv, x[3] * inv};
    uint8_t* cache = static_cast<uint8_t*>(is_k ? a.k_cache : a.v_cache);
    *reinterpret_cast<uint32_t*>(cache + dst) = f32x4_to_e4m3(q);
  }
}

cudaError_t launch_qkv_post(const void* qkv, int64_t qkv_stride, void* q_out, const void* q_norm, const void* k_norm,
                            float eps, const int* positions, const float* cos_sin, void* k_cache, void* v_cache,
                            float* k_scale, float* v_scale, const int* slots, int T, int nq, int nkv, int head_dim,
                            int block_size, int kv_fp8, cudaStream_t stream, int num_blocks) {
  if (T == 0) return cudaSuccess;
  if (head_dim != HD) return cudaErrorInvalidValue;
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
