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
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace nvb {

__device__ int g_sample_error = 0;  // 300+: a vocab-parallel exchange timed out

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
__global__ void __launch_bounds__(256, 4) sample_partial_kernel(const T* __restrict__ logits, int64_t ld, int V,
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
  if (VEC && (((uintptr_t)(lr + c0)) & 15) == 0) {
    const int nv = (c1 - c0) >> 3;
    const uint4* src = reinterpret_cast<const uint4*>(lr + c0);
    const int nb = blockDim.x;
    int i = threadIdx.x;
    if (greedy) {
      // Four independent 16-byte loads in flight per thread (one at a time left each SM with about
      // 20 KB in flight, under half of what HBM needs).  The 8 values of a load are reduced with
      // bf16x2 max first; only a load whose maximum beats the running one is searched for the
      // column (a thread visits its columns in increasing order, so the first maximum wins ties).
      for (; i < nv; i += 4 * nb) {
        uint4 r[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (i + k * nb < nv) r[k] = __ldg(src + i + k * nb);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (i + k * nb >= nv) break;
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r[k]);
          const __nv_bfloat162 m2 = __hmax2(__hmax2(h[0], h[1]), __hmax2(h[2], h[3]));
          const float m = fmaxf(__low2float(m2), __high2float(m2));
          if (m > best) {
            float f[8];
            bf16x8_to_f32(r[k], f);
            int j = 0;
            while (j < 7 && f[j] != m) ++j;
            best = m;
            bidx = c0 + (i + k * nb) * 8 + j;
          }
        }
      }
    } else {
      for (; i < nv; i += nb) {
        float f[8];
        bf16x8_to_f32(__ldg(src + i), f);
        const int cb = c0 + i * 8;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          consider(noised(f[j], inv_t, seed, step, row, col_offset + cb + j), cb + j, best, bidx);
      }
    }
    for (int c = c0 + nv * 8 + threadIdx.x; c < c1; c += nb) {
      float v = to_f<T>(lr[c]);
      if (!greedy) v = noised(v, inv_t, seed, step, row, col_offset + c);
      consider(v, c, best, bidx);
    }
  } else {
    for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
      float v = to_f<T>(lr[c]);
      if (!greedy) v = noised(v, inv_t, seed, step, row, col_offset + c);
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

// Tokens from the keys of the lm_head GEMM's sampling epilogue (orderable score << 32 | ~column);
// every key is zeroed again for the next launch.  A row whose key stayed zero (no finite score)
// gets token 0, as the chunked sampler gives it.
__global__ void sample_keys_kernel(unsigned long long* __restrict__ keys, int rows, int* __restrict__ out_tok,
                                   float* __restrict__ out_val) {
  pdl_wait();     // the keys come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows) return;
  const unsigned long long k = keys[i];
  keys[i] = 0ull;
  if (k == 0ull) {
    out_tok[i] = 0;
    if (out_val) out_val[i] = -INFINITY;
    return;
  }
  out_tok[i] = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
  if (out_val) {
    const uint32_t u = (uint32_t)(k >> 32);
    out_val[i] = __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
  }
}

cudaError_t launch_sample_keys(unsigned long long* keys, int rows, int* out_tok, float* out_val, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  launch_pdl(sample_keys_kernel, dim3((rows + 255) / 256), dim3(256), 0, stream, keys, rows, out_tok, out_val);
  NVB_LAUNCH_CHECK();
  return cudaSuccess;
}

int sample_num_chunks(int rows, int V) {
  // at most 4 CTAs per SM in total (the partial kernel's residency), so every CTA runs in the first
  // wave; chunks of at least 4096 columns (a multiple of 8, so every chunk of a 16-byte-aligned row
  // starts aligned)
  int want = (4 * 148) / (rows > 0 ? rows : 1);
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



// ------------------------------------------------------------------ row-parallel sampler
// One CTA per row: greedy, temperature (Gumbel-max) and nucleus (top-p) sampling over this
// rank's vocabulary shard, with the cross-rank combination done inside the kernel through
// symmetric memory when the vocabulary is split over a tensor-parallel group (world > 1):
// each step's per-row values are stored into every rank's exchange area (NVLink peer
// stores), followed by a per-(row, round) flag; a CTA only ever waits for the same row's
// CTA on the other ranks, and the launch keeps every CTA resident (rows <= capacity).
//
// Top-p (nucleus) without sorting: with z = logit / T, M = max z over the whole vocabulary
// and d = M - z, the nucleus is {d < d*} for the smallest d* whose softmax mass reaches p.
//   pass 1: M (max over ranks);
//   pass 2: Z = sum exp(-d) and a histogram of exp(-d) over SAMPLE_NB bins of d in [0, 32)
//            (bins of 1/32; columns beyond d = 32 carry < 1e-13 of the mass each);
//   pass 3: the bin where the cumulative mass crosses p Z is split again into SAMPLE_NB
//            sub-bins (resolution 1/32768 in d, a probability ratio of 1.00003: ties);
//   pass 4: Gumbel-max over the nucleus (argmax of z + g over d < d*), which samples the
//            renormalised nucleus distribution, then the (score, token) pairs of the ranks.
// Greedy and plain temperature rows skip passes 1-3.
namespace {

__device__ __forceinline__ uint32_t sx_ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t sx_ld_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void sx_st_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}


// Float offsets of the exchange regions and word offsets of the flags (see SampleX).
__device__ __forceinline__ int64_t sx_region(const SampleX& X, int round) {
  const int64_t wr = (int64_t)X.world * X.rows_cap;
  switch (round) {
    case 1: return 0;
    case 2: return wr;
    case 3: return wr + wr * (SAMPLE_NB + 1);
    default: return wr + wr * (SAMPLE_NB + 1) + wr * SAMPLE_NB;
  }
}
__device__ __forceinline__ int sx_width(int round) {
  return round == 1 ? 1 : round == 2 ? SAMPLE_NB + 1 : round == 3 ? SAMPLE_NB : 2;
}

// Publish `vals` (n floats, shared memory) of this row for round `round` at every rank, then
// wait until every rank published its own; returns false (error word set) on timeout.
__device__ bool sx_exchange(const SampleX& X, int round, int row, const float* vals, uint32_t epoch, bool* ok_s) {
  const int n = sx_width(round);
  const int64_t off = sx_region(X, round) + ((int64_t)X.rank * X.rows_cap + row) * n;
  for (int p = 0; p < X.world; ++p)
    for (int i = threadIdx.x; i < n; i += blockDim.x) X.x[p][off + i] = vals[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    const int64_t fo = ((int64_t)(round - 1) * X.rows_cap + row) * X.world;
    for (int p = 0; p < X.world; ++p) sx_st_sys(X.f[p] + fo + X.rank, epoch);
    const uint32_t* mine = X.f[X.rank] + fo;
    SpinBudget sb;
    bool ok = true;
    for (int p = 0; p < X.world && ok; ++p) {
      while ((int32_t)(sx_ld_sys(mine + p) - epoch) < 0) {
        if (sb.expired(X.timeout_ns)) {
          atomicCAS(&g_sample_error, 0, 300 + round);
          ok = false;
          break;
        }
      }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    *ok_s = ok;
  }
  __syncthreads();
  return *ok_s;
}

// Value i of rank p's round-`round` contribution for this row (written by peers: bypass L1).
__device__ __forceinline__ float sx_get(const SampleX& X, int round, int row, int p, int i) {
  const int n = sx_width(round);
  return __ldcv(X.x[X.rank] + sx_region(X, round) + ((int64_t)p * X.rows_cap + row) * n + i);
}

__device__ __forceinline__ float block_reduce_max(float v, float* red) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : -INFINITY;
    t = warp_max(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

// First bin whose cumulative mass (from bin 0) reaches `target`, given `base` mass before
// bin 0; *before = cumulative mass before that bin.  Single warp (warp 0), SAMPLE_NB bins.
__device__ __forceinline__ int find_cut(const float* hist, float base, float target, float* before) {
  const int lane = threadIdx.x & 31;
  constexpr int PER = SAMPLE_NB / 32;
  float local[PER];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    local[i] = hist[lane * PER + i];
    s += local[i];
  }
  // exclusive prefix over lanes
  float incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(FULL_MASK, incl, o);
    if (lane >= o) incl += t;
  }
  float run = base + incl - s;
  int cut = SAMPLE_NB;  // not reached: everything below the window
  float bef = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    if (cut == SAMPLE_NB && run + local[i] >= target) {
      cut = lane * PER + i;
      bef = run;
    }
    run += local[i];
  }
  // smallest lane with a hit
  const unsigned hit = __ballot_sync(FULL_MASK, cut != SAMPLE_NB);
  if (!hit) {
    *before = base + __shfl_sync(FULL_MASK, incl, 31);
    return SAMPLE_NB;
  }
  const int src = __ffs(hit) - 1;
  *before = __shfl_sync(FULL_MASK, bef, src);
  return __shfl_sync(FULL_MASK, cut, src);
}

template <typename T>
__global__ void __launch_bounds__(1024) sample_rows_kernel(const T* __restrict__ logits, int64_t ld, int V,
                                                           int64_t col_offset, const float* __restrict__ temps,
                                                           const float* __restrict__ top_p,
                                                           const int64_t* __restrict__ seed_step,
                                                           int* __restrict__ out_tok, float* __restrict__ out_val,
                                                           int rows, SampleX X) {
  pdl_wait();
  pdl_trigger();
  __shared__ float hist[SAMPLE_NB + 1];
  __shared__ float red[32];
  __shared__ float sval[2];
  __shared__ uint32_t s_epoch;
  __shared__ bool s_ok;
  __shared__ float s_cut;
  const uint64_t seed = (uint64_t)seed_step[0], step = (uint64_t)seed_step[1];
  const bool multi = X.world > 1;
  if (threadIdx.x == 0) s_epoch = multi ? sx_ld_acquire(X.ctrl) + 1 : 0u;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  bool ok = true;  // false after a failed exchange: later rows are sampled from this shard alone
  // CTA b samples rows b, b + grid, ...: the same rows in the same order on every rank, so with
  // every CTA resident each exchange finds its peer CTA running
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
  const float t = temps[row];
  const bool greedy = !(t > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / t;
  const float p = top_p ? top_p[row] : 1.f;
  const bool use_p = !greedy && p < 1.f;
  const T* lr = logits + (int64_t)row * ld;
  float cut_d = INFINITY, M = 0.f;
  if (use_p) {
    float m = -INFINITY;
    for (int c = threadIdx.x; c < V; c += blockDim.x) m = fmaxf(m, to_f<T>(lr[c]) * inv_t);
    M = block_reduce_max(m, red);
    if (multi) {
      if (threadIdx.x == 0) sval[0] = M;
      __syncthreads();
      ok = sx_exchange(X, 1, row, sval, epoch, &s_ok);
      if (ok && threadIdx.x == 0) {
        float g = -INFINITY;
        for (int q = 0; q < X.world; ++q) g = fmaxf(g, sx_get(X, 1, row, q, 0));
        red[0] = g;
      }
      __syncthreads();
      M = red[0];
      __syncthreads();
    }
    // pass 2: mass histogram over d = M - z in [0, 32)
    for (int i = threadIdx.x; i <= SAMPLE_NB; i += blockDim.x) hist[i] = 0.f;
    __syncthreads();
    float zl = 0.f;
    for (int c = threadIdx.x; c < V; c += blockDim.x) {
      const float d = M - to_f<T>(lr[c]) * inv_t;
      const float e = expf(-d);
      zl += e;
      if (d < 32.f) atomicAdd(&hist[min(SAMPLE_NB - 1, (int)(d * (SAMPLE_NB / 32.f)))], e);
    }
    const float Z = block_reduce_sum(zl, red);
    if (threadIdx.x == 0) hist[SAMPLE_NB] = Z;
    __syncthreads();
    if (multi && ok) {
      ok = sx_exchange(X, 2, row, hist, epoch, &s_ok);
      if (ok) {
        for (int i = threadIdx.x; i <= SAMPLE_NB; i += blockDim.x) {
          float s = 0.f;
          for (int q = 0; q < X.world; ++q) s += sx_get(X, 2, row, q, i);
          hist[i] = s;
        }
      }
      __syncthreads();
    }
    const float target = p * hist[SAMPLE_NB];
    __shared__ int s_b1;
    __shared__ float s_before;
    if (threadIdx.x < 32) {
      float before;
      const int b1 = find_cut(hist, 0.f, target, &before);
      if (threadIdx.x == 0) {
        s_b1 = b1;
        s_before = before;
      }
    }
    __syncthreads();
    const int b1 = s_b1;
    const float before = s_before;
    if (b1 >= SAMPLE_NB) {
      cut_d = 32.f;  // the mass reaches p only with the far tail: keep the whole window
    } else {
      // pass 3: split bin b1
      __syncthreads();
      for (int i = threadIdx.x; i < SAMPLE_NB; i += blockDim.x) hist[i] = 0.f;
      __syncthreads();
      const float lo = b1 * (32.f / SAMPLE_NB);
      for (int c = threadIdx.x; c < V; c += blockDim.x) {
        const float d = M - to_f<T>(lr[c]) * inv_t;
        if (d < 32.f && min(SAMPLE_NB - 1, (int)(d * (SAMPLE_NB / 32.f))) == b1) {
          const int sb = min(SAMPLE_NB - 1, max(0, (int)((d - lo) * (SAMPLE_NB * SAMPLE_NB / 32.f))));
          atomicAdd(&hist[sb], expf(-d));
        }
      }
      __syncthreads();
      if (multi && ok) {
        ok = sx_exchange(X, 3, row, hist, epoch, &s_ok);
        if (ok) {
          for (int i = threadIdx.x; i < SAMPLE_NB; i += blockDim.x) {
            float s = 0.f;
            for (int q = 0; q < X.world; ++q) s += sx_get(X, 3, row, q, i);
            hist[i] = s;
          }
        }
        __syncthreads();
      }
      if (threadIdx.x < 32) {
        float b2before;
        const int b2 = find_cut(hist, before, target, &b2before);
        if (threadIdx.x == 0)
          s_cut = b2 >= SAMPLE_NB ? lo + 32.f / SAMPLE_NB : lo + (b2 + 1) * (32.f / SAMPLE_NB / SAMPLE_NB);
      }
      __syncthreads();
      cut_d = s_cut;
    }
  }
  // argmax of the (noised) scores over this shard's admitted columns
  float best = -INFINITY;
  int bidx = 0x7fffffff;
  for (int c = threadIdx.x; c < V; c += blockDim.x) {
    const float l = to_f<T>(lr[c]);
    if (use_p && M - l * inv_t >= cut_d) continue;
    const float v = greedy ? l : noised(l, inv_t, seed, step, row, col_offset + c);
    consider(v, c, best, bidx);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(FULL_MASK, best, o);
    const int oi = __shfl_xor_sync(FULL_MASK, bidx, o);
    if (ov > best || (ov == best && oi < bidx)) {
      best = ov;
      bidx = oi;
    }
  }
  __shared__ float wv[32];
  __shared__ int wi[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    wv[w] = best;
    wi[w] = bidx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i)
      if (wv[i] > best || (wv[i] == best && wi[i] < bidx)) {
        best = wv[i];
        bidx = wi[i];
      }
    const int64_t gidx = bidx == 0x7fffffff ? -1 : (int64_t)bidx + col_offset;
    sval[0] = best;
    sval[1] = __int_as_float((int)gidx);
  }
  __syncthreads();
  if (multi && ok) {
    ok = sx_exchange(X, 4, row, sval, epoch, &s_ok);
    if (threadIdx.x == 0 && ok) {
      float b = -INFINITY;
      int bi = 0x7fffffff;
      for (int q = 0; q < X.world; ++q) {
        const float v = sx_get(X, 4, row, q, 0);
        const int i = __float_as_int(sx_get(X, 4, row, q, 1));
        if (i >= 0 && (v > b || (v == b && i < bi))) {
          b = v;
          bi = i;
        }
      }
      sval[0] = b;
      sval[1] = __int_as_float(bi == 0x7fffffff ? -1 : bi);
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const int tok = __float_as_int(sval[1]);
    out_tok[row] = tok < 0 ? 0 : tok;
    if (out_val) out_val[row] = sval[0];
  }
  __syncthreads();  // the next row rewrites the shared buffers
  }
  if (multi && threadIdx.x == 0) {
    // the last CTA of this rank advances the call number (every CTA read it at its start)
    uint32_t prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(X.ctrl + 1) : "memory");
    if (prev == gridDim.x - 1) {
      X.ctrl[1] = 0;
      asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(X.ctrl), "r"(epoch) : "memory");
    }
  }
}

}  // namespace

int sample_rows_capacity() {
  static std::atomic<int> cached[64];  // per device; 0 = not yet computed
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64) {
    const int c = cached[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, sample_rows_kernel<__nv_bfloat16>, 1024, 0) != cudaSuccess ||
      n <= 0) {
    cudaGetLastError();
    n = 1;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < 64) cached[dev].store(n * sms, std::memory_order_relaxed);
  return n * sms;
}

cudaError_t launch_sample_rows(const void* logits, int logits_is_bf16, int64_t ld, int rows, int V, int64_t col_offset,
                               const float* temps, const float* top_p, const int64_t* seed_step, int* out_tok,
                               float* out_val, const SampleX& X, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  int grid = rows;
  if (X.world > 1) {
    if (X.world > 8 || X.rank < 0 || X.rank >= X.world || rows > X.rows_cap || !X.ctrl) return cudaErrorInvalidValue;
    for (int p = 0; p < X.world; ++p)
      if (!X.x[p] || !X.f[p]) return cudaErrorInvalidValue;
    // every CTA waits for its rows on the other ranks: all of them must be resident
    const int cap = sample_rows_capacity();
    if (grid > cap) grid = cap;
  }
  if (logits_is_bf16)
    launch_pdl(sample_rows_kernel<__nv_bfloat16>, dim3(grid), dim3(1024), 0, stream,
               static_cast<const __nv_bfloat16*>(logits), ld, V, col_offset, temps, top_p, seed_step, out_tok, out_val,
               rows, X);
  else
    launch_pdl(sample_rows_kernel<float>, dim3(grid), dim3(1024), 0, stream, static_cast<const float*>(logits), ld, V,
               col_offset, temps, top_p, seed_step, out_tok, out_val, rows, X);
  NVB_LAUNCH_CHECK();
  return cudaSuccess;
}

int sample_error_code(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_sample_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_sample_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace nvb
