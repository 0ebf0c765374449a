// Greedy / temperature sampling over (possibly vocab-sharded) logits via the Gumbel-max rule.
//
// Reference: nanovllm/layers/sampler.py:9-43 (argmax when temperature <= 0, otherwise
// softmax(logits / T) + multinomial).  Sampling from softmax(l / T) equals taking
// argmax(l / T + g) with g i.i.d. Gumbel(0, 1) noise (the Gumbel-max trick, Gumbel 1954;
// Maddison et al. 2014), which needs no normalisation and splits over vocab shards: a
// shard reports (max, argmax) of its columns and the shards' maxima are compared.
// The noise for (row, global column) comes from a counter-based hash of (seed, step,
// row, column) (SplitMix64 finaliser, Steele et al. 2014), so every TP rank draws the
// same noise for the same column and the whole sampler is CUDA-graph safe.
#include "common.cuh"
#include "kernels.h"

namespace nvb {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ float gumbel(uint64_t seed, uint64_t step, int row, int64_t col) {
  uint64_t h = mix64(seed + 0x9E3779B97F4A7C15ull * (step + 1));
  h = mix64(h ^ ((uint64_t)row << 40) ^ (uint64_t)col);
  float u = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
  return -logf(-logf(u));
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ void consider(float v, int c, float& best, int& bidx) {
  if (v > best || (v == best && c < bidx)) {
    best = v;
    bidx = c;
  }
}

// Partial (max, argmax) of the noised scores over one column chunk of one row.  bf16
// rows are read 8 columns per 16-byte load when the row start is 16-byte aligned.
template <typename T>
__global__ void __launch_bounds__(256) sample_partial_kernel(const T* __restrict__ logits, int64_t ld, int V,
                                                             int64_t col_offset, const float* __restrict__ temps,
                                                             const int64_t* __restrict__ seed_step,
                                                             float* __restrict__ part_val, int* __restrict__ part_idx,
                                                             int chunk) {
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  const int row = blockIdx.y, ch = blockIdx.x;
  const float t = temps[row];
  const bool greedy = !(t > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / t;
  const uint64_t seed = (uint64_t)seed_step[0], step = (uint64_t)seed_step[1];
  const int c0 = ch * chunk, c1 = min(V, c0 + chunk);
  float best = -INFINITY;
  int bidx = 0x7fffffff;
  const T* lr = logits + (int64_t)row * ld;
  constexpr bool VEC = sizeof(T) == 2;
  if (VEC && (((uintptr_t)(lr + c0)) & 15) == 0 && greedy) {
    const int nv = (c1 - c0) >> 3;
    const uint4* src = reinterpret_cast<const uint4*>(lr + c0);
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      float f[8];
      bf16x8_to_f32(__ldg(src + i), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) consider(f[j], c0 + i * 8 + j, best, bidx);
    }
    for (int c = c0 + nv * 8 + threadIdx.x; c < c1; c += blockDim.x) consider(to_f<T>(lr[c]), c, best, bidx);
  } else if (VEC && (((uintptr_t)(lr + c0)) & 15) == 0) {
    const int nv = (c1 - c0) >> 3;
    const uint4* src = reinterpret_cast<const uint4*>(lr + c0);
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      float f[8];
      bf16x8_to_f32(__ldg(src + i), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = c0 + i * 8 + j;
        consider(f[j] * inv_t + gumbel(seed, step, row, col_offset + c), c, best, bidx);
      }
    }
    for (int c = c0 + nv * 8 + threadIdx.x; c < c1; c += blockDim.x)
      consider(to_f<T>(lr[c]) * inv_t + gumbel(seed, step, row, col_offset + c), c, best, bidx);
  } else {
    for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
      float v = to_f<T>(lr[c]);
      if (!greedy) v = v * inv_t + gumbel(seed, step, row, col_offset + c);
      consider(v, c, best, bidx);
    }
  }
  __shared__ float sv[8];
  __shared__ int si[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(FULL_MASK, best, o);
    int oi = __shfl_xor_sync(FULL_MASK, bidx, o);
    if (ov > best || (ov == best && oi < bidx)) {
      best = ov;
      bidx = oi;
    }
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    sv[w] = best;
    si[w] = bidx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i)
      if (sv[i] > best || (sv[i] == best && si[i] < bidx)) {
        best = sv[i];
        bidx = si[i];
      }
    part_val[(int64_t)row * gridDim.x + ch] = best;
    part_idx[(int64_t)row * gridDim.x + ch] = bidx == 0x7fffffff ? 0 : (int)(bidx + col_offset);
  }
}

// One warp per row: reduce the chunk partials; writes the token id and the winning score.
__global__ void sample_final_kernel(const float* __restrict__ part_val, const int* __restrict__ part_idx, int nchunk,
                                    int rows, int* __restrict__ out_tok, float* __restrict__ out_val) {
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float best = -INFINITY;
  int bidx = 0x7fffffff;
  for (int c = lane; c < nchunk; c += 32) {
    float v = part_val[(int64_t)row * nchunk + c];
    int i = part_idx[(int64_t)row * nchunk + c];
    if (v > best || (v == best && i < bidx)) {
      best = v;
      bidx = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(FULL_MASK, best, o);
    int oi = __shfl_xor_sync(FULL_MASK, bidx, o);
    if (ov > best || (ov == best && oi < bidx)) {
      best = ov;
      bidx = oi;
    }
  }
  if (lane == 0) {
    out_tok[row] = bidx == 0x7fffffff ? 0 : bidx;
    if (out_val) out_val[row] = best;
  }
}

int sample_num_chunks(int rows, int V) {
  // ~4 CTAs per SM in total, chunks of at least 4096 columns (a multiple of 8, so every
  // chunk of a 16-byte-aligned row starts aligned)
  int want = (4 * 148 + rows - 1) / (rows > 0 ? rows : 1);
  int max_chunks = (V + 4095) / 4096;
  int n = want < max_chunks ? want : max_chunks;
  return n < 1 ? 1 : n;
}

cudaError_t launch_sample(const void* logits, int logits_is_bf16, int64_t ld, int rows, int V, int64_t col_offset,
                          const float* temps, const int64_t* seed_step, float* part_val, int* part_idx, int nchunk,
                          int* out_tok, float* out_val, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  int chunk = (V + nchunk - 1) / nchunk;
  chunk = (chunk + 7) & ~7;
  dim3 grid(nchunk, rows);
  if (logits_is_bf16)
    launch_pdl(sample_partial_kernel<__nv_bfloat16>, grid, dim3(256), 0, stream,
               static_cast<const __nv_bfloat16*>(logits), ld, V, col_offset, temps, seed_step, part_val, part_idx, chunk);
  else
    launch_pdl(sample_partial_kernel<float>, grid, dim3(256), 0, stream, static_cast<const float*>(logits), ld, V,
               col_offset, temps, seed_step, part_val, part_idx, chunk);
  NVB_LAUNCH_CHECK();
  launch_pdl(sample_final_kernel, dim3((rows + 3) / 4), dim3(128), 0, stream, part_val, part_idx, nchunk, rows, out_tok,
             out_val);
  NVB_LAUNCH_CHECK();
  return cudaSuccess;
}

}  // namespace nvb
