// Residual-add + RMSNorm, SiLU-and-mul, and vocab-sharded embedding gather (bf16).
//
// Reference ops replaced: RMSNorm (nanovllm/layers/RMSNorm.py:11-17, five eager
// kernels per call), the residual adds around it (nanovllm/models/qwen3.py:126,140),
// silu(gate)*up (qwen3.py:133) and nn.Embedding (qwen3.py:483).
#include "common.cuh"
#include "kernels.h"

namespace nvb {

__device__ int g_norm_check = 0;  // bounds-check word of this file (401: gathered row out of range)

int bounds_check_enabled() { return NVB_BOUNDS_CHECK; }

int norm_check_code(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_norm_check, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_norm_check, &z, sizeof(int));
  }
  return v;
}

// One CTA per output row.  residual_out = x + residual_in (rounded to bf16, as an
// eager bf16 add would be); out = rmsnorm(residual_out) * w.  residual_in == nullptr
// means the residual is x itself and nothing is written to residual_out.  With
// row_index, output row r reads input row row_index[r] of x and residual_in (the final
// norm runs only on the rows that are sampled).
template <int NI>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride,
                                                          const __nv_bfloat16* residual_in, __nv_bfloat16* residual_out,
                                                          const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                                          int H, float eps, const int* __restrict__ row_index,
                                                          int src_rows) {
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  const int row = blockIdx.x;
  const int src_row = row_index ? row_index[row] : row;
  if (row_index && !in_range(src_row, src_rows, &g_norm_check, 401)) return;  // uniform over the CTA
  const int nvec = H >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)src_row * x_stride);
  float v[NI][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    int c = threadIdx.x + i * blockDim.x;
    if (c < nvec) {
      bf16x8_to_f32(xr[c], v[i]);
      if (residual_in) {
        float r[8];
        bf16x8_to_f32(reinterpret_cast<const uint4*>(residual_in + (int64_t)src_row * H)[c], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = bf16_round(v[i][j] + r[j]);
        reinterpret_cast<uint4*>(residual_out + (int64_t)row * H)[c] = f32_to_bf16x8(v[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) red[wid] = ss;
  __syncthreads();
  if (wid == 0) {
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) red[0] = rsqrtf(t / (float)H + eps);
  }
  __syncthreads();
  const float inv = red[0];
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* orow = reinterpret_cast<uint4*>(out + (int64_t)row * H);
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    int c = threadIdx.x + i * blockDim.x;
    if (c < nvec) {
      float wf[8], o[8];
      bf16x8_to_f32(wr[c], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * inv * wf[j];
      orow[c] = f32_to_bf16x8(o);
    }
  }
}

cudaError_t launch_add_rmsnorm(const void* x, int64_t x_stride, const void* residual_in, void* residual_out,
                               const void* w, void* out, int rows, int H, float eps, const int* row_index,
                               cudaStream_t stream, int src_rows) {
  if (rows == 0) return cudaSuccess;
  if (H % 8 != 0 || H > 8 * 256 * 4) return cudaErrorInvalidValue;
  int nvec = H / 8;
  int threads = nvec >= 256 ? 256 : ((nvec + 31) / 32) * 32;
  int ni = (nvec + threads - 1) / threads;
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto R = static_cast<const __nv_bfloat16*>(residual_in);
  auto RO = static_cast<__nv_bfloat16*>(residual_out);
  auto W = static_cast<const __nv_bfloat16*>(w);
  auto O = static_cast<__nv_bfloat16*>(out);
  switch (ni) {
    case 1: launch_pdl(add_rmsnorm_kernel<1>, dim3(rows), dim3(threads), 0, stream, X, x_stride, R, RO, W, O, H, eps, row_index, src_rows); break;
    case 2: launch_pdl(add_rmsnorm_kernel<2>, dim3(rows), dim3(threads), 0, stream, X, x_stride, R, RO, W, O, H, eps, row_index, src_rows); break;
    case 3: launch_pdl(add_rmsnorm_kernel<3>, dim3(rows), dim3(threads), 0, stream, X, x_stride, R, RO, W, O, H, eps, row_index, src_rows); break;
    default: launch_pdl(add_rmsnorm_kernel<4>, dim3(rows), dim3(threads), 0, stream, X, x_stride, R, RO, W, O, H, eps, row_index, src_rows); break;
  }
  NVB_LAUNCH_CHECK();
  return cudaSuccess;
}

// out[t, c] = silu(x[t, c]) * x[t, I + c]; 8 columns per thread.
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ out, int T, int I) {
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  const int64_t nvec_row = I >> 3;
  const int64_t total = (int64_t)T * nvec_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = i / nvec_row, c = i - t * nvec_row;
    const uint4* row = reinterpret_cast<const uint4*>(x + t * 2 * I);
    float g[8], u[8], o[8];
    bf16x8_to_f32(row[c], g);
    bf16x8_to_f32(row[nvec_row + c], u);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = g[j] / (1.f + expf(-g[j])) * u[j];
    reinterpret_cast<uint4*>(out + t * I)[c] = f32_to_bf16x8(o);
  }
}

cudaError_t launch_silu_mul(const void* x, void* out, int T, int I, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (I % 8) return cudaErrorInvalidValue;
  int64_t total = (int64_t)T * (I / 8);
  int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  silu_mul_kernel<<<(int)blocks, threads, 0, stream>>>(static_cast<const __nv_bfloat16*>(x),
                                                       static_cast<__nv_bfloat16*>(out), T, I);
  NVB_LAUNCH_CHECK();
  return cudaSuccess;
}

// Rows of a vocab shard [vocab_start, vocab_start + rows); other ids produce zeros.
__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table, int rows,
                                 int vocab_start, __nv_bfloat16* __restrict__ out, int H) {
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  const int t = blockIdx.x;
  const int local = ids[t] - vocab_start;
  const int nvec = H >> 3;
  uint4* o = reinterpret_cast<uint4*>(out + (int64_t)t * H);
  if (local < 0 || local >= rows) {
    for (int c = threadIdx.x; c < nvec; c += blockDim.x) o[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + (int64_t)local * H);
  for (int c = threadIdx.x; c < nvec; c += blockDim.x) o[c] = src[c];
}

cudaError_t launch_embedding(const int* ids, const void* table, int rows, int vocab_start, void* out, int T, int H,
                             cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (H % 8) return cudaErrorInvalidValue;
  embedding_kernel<<<T, 128, 0, stream>>>(ids, static_cast<const __nv_bfloat16*>(table), rows, vocab_start,
                                          static_cast<__nv_bfloat16*>(out), H);
  NVB_LAUNCH_CHECK();
  return cudaSuccess;
}

}  // namespace nvb
