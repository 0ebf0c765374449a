// Shared device helpers for the sm_100a kernels of nanovllm_self_b200.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include <atomic>

// Index checks on the scattered accesses whose indices come from the host (KV slots, gathered
// rows).  On (the default) every such index is range-checked; a bad one records an error code
// in the kernel file's check word (read with bounds_error) and the access is skipped, so a bad
// index never faults the GPU.  Building with -DNVB_BOUNDS_CHECK=0 removes the checks.
#ifndef NVB_BOUNDS_CHECK
#define NVB_BOUNDS_CHECK 1
#endif

namespace nvb {

constexpr unsigned FULL_MASK = 0xffffffffu;

// True when 0 <= i < n; otherwise records `code` in *word (first error wins) and returns false.
__device__ __forceinline__ bool in_range(long long i, long long n, int* word, int code) {
#if NVB_BOUNDS_CHECK
  if (i < 0 || i >= n) {
    atomicCAS(word, 0, code);
    return false;
  }
#endif
  return true;
}

// One lane of a converged warp (elect.sync): the issuing lane of a warp that runs a loop together.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile("{\n .reg .pred P;\n elect.sync _|P, 0xffffffff;\n selp.u32 %0, 1, 0, P;\n}\n" : "=r"(pred));
  return pred != 0;
}

// Time bound for a polling loop: call expired() once per failed poll.  %globaltimer is read only
// on every 64th call (a timer read costs far more than a poll of an mbarrier or a flag, and a
// read per poll slows the detection of the awaited event); true once more than budget_ns have
// passed since the first read.
struct SpinBudget {
  uint64_t t0 = 0;
  uint32_t n = 0;
  __device__ __forceinline__ bool expired(uint64_t budget_ns) {
    if ((++n & 63u) != 0) return false;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t0 == 0) {
      t0 = t;
      return false;
    }
    return t - t0 > budget_ns;
  }
};

// Gumbel-max sampling noise, shared by the sampler kernels and the lm_head GEMM's sampling
// epilogue so that both draw the same noise for (seed, step, row, global column).
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ float gumbel(uint64_t seed, uint64_t step, int row, int64_t col) {
  uint64_t h = mix64(seed + 0x9E3779B97F4A7C15ull * (step + 1));
  h = mix64(h ^ ((uint64_t)row << 40) ^ (uint64_t)col);
  // 23 random bits: (k + 0.5) / 2^23 is exact in fp32 and lies in [2^-24, 1 - 2^-24], so u < 1 and
  // the noise is finite (24 bits would round the top value up to u = 1 and give g = +inf,
  // letting a random column win about once per 2^24 columns)
  const float u = ((float)(h >> 41) + 0.5f) * (1.0f / 8388608.0f);
  return -logf(-logf(u));
}

// Noised score of a logit at temperature 1 / inv_t: l * inv_t + g, rounded once (explicit fma, so
// every kernel that computes it gets the same bits).
__device__ __forceinline__ float noised(float l, float inv_t, uint64_t seed, uint64_t step, int row, int64_t col) {
  return __fmaf_rn(l, inv_t, gumbel(seed, step, row, col));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL_MASK, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL_MASK, v, o));
  return v;
}

// 8 x bf16 <-> 8 x f32 through one 16-byte vector.
__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 f32_to_bf16x8(const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

__device__ __forceinline__ void bf16x4_to_f32(const uint2& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}

__device__ __forceinline__ uint2 f32_to_bf16x4(const float* f) {
  uint2 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
  h[0] = __floats2bfloat162_rn(f[0], f[1]);
  h[1] = __floats2bfloat162_rn(f[2], f[3]);
  return u;
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// fp8 e4m3 (saturating) conversion of 4 floats packed into 32 bits.
__device__ __forceinline__ uint32_t f32x4_to_e4m3(const float* f) {
  __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(f[0], f[1]), __NV_SATFINITE, __NV_E4M3);
  __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(f[2], f[3]), __NV_SATFINITE, __NV_E4M3);
  return uint32_t(lo) | (uint32_t(hi) << 16);
}

__device__ __forceinline__ void e4m3x4_to_f32(uint32_t v, float* f) {
  __half2_raw a = __nv_cvt_fp8x2_to_halfraw2(__nv_fp8x2_storage_t(v & 0xffff), __NV_E4M3);
  __half2_raw b = __nv_cvt_fp8x2_to_halfraw2(__nv_fp8x2_storage_t(v >> 16), __NV_E4M3);
  float2 x = __half22float2(*reinterpret_cast<__half2*>(&a));
  float2 y = __half22float2(*reinterpret_cast<__half2*>(&b));
  f[0] = x.x; f[1] = x.y; f[2] = y.x; f[3] = y.y;
}

// Programmatic dependent launch.  pdl_trigger(): this CTA no longer holds back the launch
// of the next kernel in the stream (when every CTA has triggered or exited, a kernel
// launched with the programmatic-serialization attribute may start); pdl_wait(): block
// until the previous kernel in the stream has completed and its writes are visible (a
// no-op when this kernel was not launched as a programmatic dependent).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launch `kern` as a programmatic dependent of the previous kernel in the stream: it may
// start (and run up to its pdl_wait()) while that kernel is still finishing.  Every kernel
// launched this way calls pdl_wait() before touching memory the previous kernel uses.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Runs `set_up` (kernel attribute calls such as the dynamic shared-memory opt-in) once per
// device.  Kernel attributes belong to one device, so a process that launches on several GPUs
// has to set them on each; `done` is a bitmask of the devices already set up, owned by the
// caller (one per kernel).  Devices numbered 64 and above are set up on every call.  Two
// threads may both run `set_up` for the same device; the calls are idempotent.
template <typename F>
inline cudaError_t once_per_device(std::atomic<uint64_t>& done, F&& set_up) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev >= 0 && dev < 64 ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = set_up();
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// Opt `kern` in to `bytes` of dynamic shared memory on the current device (once per device).
template <typename K>
inline cudaError_t smem_opt_in(std::atomic<uint64_t>& done, K kern, int bytes, bool nonportable_cluster = false) {
  return once_per_device(done, [&]() -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && nonportable_cluster)
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    return e;
  });
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

}  // namespace nvb

#define NVB_LAUNCH_CHECK() \
  do { cudaError_t e_ = cudaGetLastError(); if (e_ != cudaSuccess) return e_; } while (0)
