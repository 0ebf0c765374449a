// Tensor-parallel all-reduce fused with residual add + RMSNorm, over NVLink peer memory.
//
// Replaces the reference's NCCL all_reduce after o_proj / down_proj
// (nanovllm/distributed/parallel_state.py:62-71, called at nanovllm/models/qwen3.py:124,138)
// together with the residual add and the next RMSNorm (qwen3.py:126-129, :140 + next ln1).
//
// Symmetric buffers (one cudaMalloc per rank, opened by every peer through CUDA IPC):
//   IN  [rows, H] bf16  per-rank partial sums (the row-parallel GEMM writes here)
//   RES [rows, H] bf16  residual stream (replicated)
//   OUT [rows, H] bf16  RMSNorm output (replicated; the next GEMM reads it)
//   FLAGS               cross-rank barrier flags + local control words (comm.h)
// Two-shot algorithm, one launch, grid = NCTA CTAs on every rank:
//   1. barrier A: CTA 0 tells every peer "my IN is ready" (the GEMM that wrote IN
//      precedes this kernel on each rank's stream), waits for the peers, and releases the
//      other CTAs of its rank through a local go word;
//   2. rank r owns rows [r*T/tp, (r+1)*T/tp); CTA b takes every NCTA-th owned row,
//      sums the row over all peers' IN (NVLink loads), adds RES, normalises, and stores
//      the new RES row and the OUT row into every rank's buffers (NVLink stores);
//   3. barrier B: the last CTA of the rank to finish tells every peer "all my stores are
//      done" and waits for the peers before it exits, so when the kernel completes every
//      rank holds all rows of RES and OUT.
// Barriers are per rank (one NVLink round trip per call, whatever the CTA count).  The
// call number lives in device memory and is advanced by the kernel itself, so the call is
// CUDA-graph capturable.  Every wait is bounded by a wall-clock budget; on expiry the
// kernel records an error code (read with comm_error_code) and returns.
#include <cuda_runtime.h>

#include "comm.h"
#include "common.cuh"

namespace nvb {

__device__ int g_comm_error = 0;

namespace {

constexpr uint64_t COMM_WAIT_NS = 10000000000ull;  // default 10 s: ranks may autotune GEMMs at different speeds

__device__ __forceinline__ uint64_t wait_budget(const CommArgs& a) {
  return a.timeout_ns ? a.timeout_ns : COMM_WAIT_NS;
}


__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wraparound-safe "flag has reached call e".
__device__ __forceinline__ bool reached(uint32_t v, uint32_t e) { return (int32_t)(v - e) >= 0; }

// Wait (one thread) until every rank's word in slot `flags_off` of this rank's flags has
// reached call number `epoch`; false (after recording `code`) when `budget_ns` runs out.
__device__ bool wait_all_flags(uint32_t* const* flags, int rank, int world, size_t flags_off, uint32_t epoch,
                               uint64_t budget_ns, int code) {
  const uint32_t* mine = flags[rank] + flags_off;
  SpinBudget sb;
  for (int p = 0; p < world; ++p) {
    while (!reached(ld_relaxed_sys(mine + p), epoch)) {
      if (sb.expired(budget_ns)) {
        atomicCAS(&g_comm_error, 0, code);
        fence_acq_rel_sys();
        return false;
      }
    }
  }
  fence_acq_rel_sys();
  return true;
}

// Cross-rank part of a per-rank barrier (one thread): publish call number `epoch` in slot
// `flags_off` of every rank, then wait until every rank published it (or a later one) here.
__device__ bool rank_exchange_raw(uint32_t* const* flags, int rank, int world, size_t flags_off, uint32_t epoch,
                                  uint64_t budget_ns, int code) {
  fence_acq_rel_sys();
  for (int p = 0; p < world; ++p) st_relaxed_sys(flags[p] + flags_off + rank, epoch);
  return wait_all_flags(flags, rank, world, flags_off, epoch, budget_ns, code);
}

__device__ bool rank_exchange(const CommArgs& a, size_t flags_off, uint32_t epoch, int code) {
  return rank_exchange_raw(a.flags, a.rank, a.world, flags_off, epoch, wait_budget(a), code);
}

// Entry barrier (thread 0 of each CTA): every CTA reads this call's number from the local
// counter; CTA 0 exchanges flags with the peers and then releases the other CTAs of this
// rank through the local go word.  All CTAs of a call are resident together (grid <= the
// SM count), so waiting on CTA 0 cannot stall.
__device__ bool rank_entry_barrier(const CommArgs& a, size_t flags_off, uint32_t& epoch) {
  uint32_t* ctrl = a.flags[a.rank] + COMM_CTRL;  // [0] calls, [1] go, [2] done, [3] go error
  epoch = ld_acquire_gpu(ctrl) + 1;
  if (blockIdx.x == 0) {
    const bool ok = rank_exchange(a, flags_off, epoch, 110);
    if (!ok) ctrl[3] = epoch;
    st_release_gpu(ctrl + 1, epoch);
    return ok;
  }
  // twice CTA 0's budget: when the peers fail to arrive, CTA 0 gives up first, records why
  // (110) and releases this CTA through the go word; 111 means CTA 0 itself never got there
  SpinBudget sb;
  while (!reached(ld_acquire_gpu(ctrl + 1), epoch)) {
    if (sb.expired(2 * wait_budget(a))) {
      atomicCAS(&g_comm_error, 0, 111);
      return false;
    }
  }
  return ld_acquire_gpu(ctrl + 3) != epoch;
}

// Exit (thread 0 of each CTA, after a __syncthreads): the last CTA of this rank to get here
// optionally runs the exit barrier with the peers, then advances the call counter.
__device__ void rank_exit(const CommArgs& a, uint32_t epoch, bool exit_barrier, bool ok) {
  uint32_t* ctrl = a.flags[a.rank] + COMM_CTRL;
  // this CTA's stores before its arrival: system scope only when they went to peers
  if (exit_barrier) fence_acq_rel_sys();
  else __threadfence();
  uint32_t prev;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(ctrl + 2) : "memory");
  if (prev != gridDim.x - 1) return;
  if (exit_barrier && ok) rank_exchange(a, COMM_TWOSHOT_B, epoch, 112);
  ctrl[2] = 0;
  st_release_gpu(ctrl, epoch);
}

template <int NI>
__global__ void __launch_bounds__(256) allreduce_add_rmsnorm_kernel(CommArgs a) {
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  const int b = blockIdx.x;
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  __shared__ float red[32];
  if (threadIdx.x == 0) {
    uint32_t e = 0;
    s_ok = rank_entry_barrier(a, COMM_TWOSHOT_A, e) ? 1 : 0;
    s_epoch = e;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  if (s_ok) {
    const int H = a.hidden;
    const int nvec = H >> 3;
    const int per = (a.rows + a.world - 1) / a.world;
    const int r0 = a.rank * per, r1 = min(a.rows, r0 + per);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    for (int row = r0 + b; row < r1; row += gridDim.x) {
      float v[NI][8];
      float ss = 0.f;
      // issue every load of the row (all peers, all vectors, the residual) before using any
      uint4 raw[NI][COMM_MAX_RANKS], rres[NI];
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        if (c < nvec) {
#pragma unroll
          for (int p = 0; p < COMM_MAX_RANKS; ++p)
            if (p < a.world) raw[i][p] = __ldcv(reinterpret_cast<const uint4*>(a.in[p] + (int64_t)row * H) + c);
          if (a.has_residual) rres[i] = reinterpret_cast<const uint4*>(a.res[a.rank] + (int64_t)row * H)[c];
        }
      }
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        if (c < nvec) {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
#pragma unroll
          for (int p = 0; p < COMM_MAX_RANKS; ++p) {
            if (p < a.world) {
              float f[8];
              bf16x8_to_f32(raw[i][p], f);
#pragma unroll
              for (int j = 0; j < 8; ++j) v[i][j] += f[j];
            }
          }
          if (a.has_residual) {
            float r[8];
            bf16x8_to_f32(rres[i], r);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i][j] = bf16_round(v[i][j] + r[j]);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i][j] = bf16_round(v[i][j]);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) red[wid] = ss;
      __syncthreads();
      if (wid == 0) {
        float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) red[0] = rsqrtf(t / (float)H + a.eps);
      }
      __syncthreads();
      const float inv = red[0];
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        if (c < nvec) {
          float wf[8], o[8];
          bf16x8_to_f32(reinterpret_cast<const uint4*>(a.weight)[c], wf);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = v[i][j] * inv * wf[j];
          const uint4 ru = f32_to_bf16x8(v[i]), ou = f32_to_bf16x8(o);
          for (int p = 0; p < a.world; ++p) {
            reinterpret_cast<uint4*>(a.res[p] + (int64_t)row * H)[c] = ru;
            reinterpret_cast<uint4*>(a.out[p] + (int64_t)row * H)[c] = ou;
          }
        }
      }
      __syncthreads();  // red[] is reused by the next row
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) rank_exit(a, epoch, true, s_ok != 0);
}

// One-shot variant for small batches: a single barrier ("every rank's IN is ready"),
// then every rank reduces ALL rows itself from the peers' IN and writes RES / OUT in its
// own memory only.  The caller rotates IN over three buffers (consecutive calls never
// share one), which is what makes the missing second barrier safe: a rank can only
// reach the barrier of call k+1 after every rank finished reading call k's buffer.
template <int NI>
__global__ void __launch_bounds__(256) allreduce_oneshot_kernel(CommArgs a) {
  pdl_wait();     // inputs come from the previous kernel in the stream
  pdl_trigger();  // the next kernel may start its prologue
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  __shared__ float red[32];
  if (threadIdx.x == 0) {
    uint32_t e = 0;
    s_ok = rank_entry_barrier(a, COMM_ONESHOT_FLAGS, e) ? 1 : 0;
    s_epoch = e;
  }
  __syncthreads();
  if (!s_ok) {
    if (threadIdx.x == 0) rank_exit(a, s_epoch, false, false);
    return;
  }
  const int b = blockIdx.x;
  const int H = a.hidden;
  const int nvec = H >> 3;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int row = b; row < a.rows; row += gridDim.x) {
    float v[NI][8];
    float ss = 0.f;
    // issue every load of the row (all peers, all of this thread's vectors, the residual)
    // before using any, so the NVLink latency is paid once per row, not once per load
    uint4 raw[NI][COMM_MAX_RANKS], rres[NI];
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nvec) {
#pragma unroll
        for (int p = 0; p < COMM_MAX_RANKS; ++p)
          if (p < a.world) raw[i][p] = __ldcv(reinterpret_cast<const uint4*>(a.in[p] + (int64_t)row * H) + c);
        if (a.has_residual) rres[i] = reinterpret_cast<const uint4*>(a.res[a.rank] + (int64_t)row * H)[c];
      }
    }
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nvec) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
#pragma unroll
        for (int p = 0; p < COMM_MAX_RANKS; ++p) {
          if (p < a.world) {
            float f[8];
            bf16x8_to_f32(raw[i][p], f);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i][j] += f[j];
          }
        }
        if (a.has_residual) {
          float r[8];
          bf16x8_to_f32(rres[i], r);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] = bf16_round(v[i][j] + r[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] = bf16_round(v[i][j]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) red[wid] = ss;
    __syncthreads();
    if (wid == 0) {
      float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
      t = warp_sum(t);
      if (lane == 0) red[0] = rsqrtf(t / (float)H + a.eps);
    }
    __syncthreads();
    const float inv = red[0];
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nvec) {
        float wf[8], o[8];
        bf16x8_to_f32(reinterpret_cast<const uint4*>(a.weight)[c], wf);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = v[i][j] * inv * wf[j];
        reinterpret_cast<uint4*>(a.res[a.rank] + (int64_t)row * H)[c] = f32_to_bf16x8(v[i]);
        reinterpret_cast<uint4*>(a.out[a.rank] + (int64_t)row * H)[c] = f32_to_bf16x8(o);
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) rank_exit(a, s_epoch, false, true);
}


// Owner side of the GEMM -> reduce-scatter path (see RsNormArgs in comm.h).  Every CTA waits
// on this rank's RS flags itself (local polling), so no CTA waits on another before the rows.
template <int NI>
__global__ void __launch_bounds__(256) rs_add_rmsnorm_ag_kernel(RsNormArgs a) {
  pdl_wait();     // the reduce-scatter GEMM before this kernel has completed on this rank
  pdl_trigger();  // the next kernel may start its prologue (its loads wait for this grid)
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  __shared__ float red[32];
  uint32_t* ctrl = a.flags[a.rank] + COMM_CTRL;
  const uint64_t budget = a.timeout_ns ? a.timeout_ns : COMM_WAIT_NS;
  if (threadIdx.x == 0) {
    const uint32_t e = ld_acquire_gpu(ctrl) + 1;
    s_epoch = e;
    s_ok = wait_all_flags(a.flags, a.rank, a.world, COMM_RS_FLAGS, e, budget, 120) ? 1 : 0;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  if (s_ok) {
    const int H = a.hidden;
    const int nvec = H >> 3;
    const int r0 = a.rank * a.rs_rows, r1 = min(a.rows, r0 + a.rs_rows);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t slot = (int64_t)COMM_RS_MAX_ROWS * H;  // elements of one source rank's slot
    for (int row = r0 + blockIdx.x; row < r1; row += gridDim.x) {
      const int lr = row - r0;
      float v[NI][8];
      float ss = 0.f;
      uint4 raw[NI][COMM_MAX_RANKS], rres[NI];
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        if (c < nvec) {
#pragma unroll
          for (int p = 0; p < COMM_MAX_RANKS; ++p)
            if (p < a.world)  // written by peers over NVLink: bypass L1
              raw[i][p] = __ldcv(reinterpret_cast<const uint4*>(a.rs + p * slot + (int64_t)lr * H) + c);
          if (a.has_residual) rres[i] = reinterpret_cast<const uint4*>(a.res + (int64_t)row * H)[c];
        }
      }
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        if (c < nvec) {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
#pragma unroll
          for (int p = 0; p < COMM_MAX_RANKS; ++p) {
            if (p < a.world) {
              float f[8];
              bf16x8_to_f32(raw[i][p], f);
#pragma unroll
              for (int j = 0; j < 8; ++j) v[i][j] += f[j];
            }
          }
          if (a.has_residual) {
            float r[8];
            bf16x8_to_f32(rres[i], r);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i][j] = bf16_round(v[i][j] + r[j]);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i][j] = bf16_round(v[i][j]);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) red[wid] = ss;
      __syncthreads();
      if (wid == 0) {
        float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) red[0] = rsqrtf(t / (float)H + a.eps);
      }
      __syncthreads();
      const float inv = red[0];
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        if (c < nvec) {
          float wf[8], o[8];
          bf16x8_to_f32(reinterpret_cast<const uint4*>(a.weight)[c], wf);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = v[i][j] * inv * wf[j];
          reinterpret_cast<uint4*>(a.res + (int64_t)row * H)[c] = f32_to_bf16x8(v[i]);
          const uint4 ou = f32_to_bf16x8(o);
          for (int p = 0; p < a.world; ++p) reinterpret_cast<uint4*>(a.out[p] + (int64_t)row * H)[c] = ou;
        }
      }
      __syncthreads();  // red[] is reused by the next row
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // this CTA's OUT stores (peers included) before its arrival; the last CTA of the rank
    // publishes "my rows are everywhere" and waits until every rank has published it
    fence_acq_rel_sys();
    uint32_t prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(ctrl + 2) : "memory");
    if (prev == gridDim.x - 1) {
      if (s_ok) rank_exchange_raw(a.flags, a.rank, a.world, COMM_AG_FLAGS, epoch, budget, 121);
      ctrl[2] = 0;
      st_release_gpu(ctrl, epoch);
    }
  }
}

}  // namespace

cudaError_t launch_rs_add_rmsnorm_ag(const RsNormArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  if (a.hidden % 8 || a.hidden > 8 * 256 * 4 || a.world > COMM_MAX_RANKS || a.world < 1 || a.ctas > COMM_MAX_CTAS ||
      a.ctas < 1 || a.rs_rows < 1 || a.rs_rows > COMM_RS_MAX_ROWS || (int64_t)a.rs_rows * a.world < a.rows)
    return cudaErrorInvalidValue;
  const int nvec = a.hidden / 8;
  const int threads = nvec >= 256 ? 256 : ((nvec + 31) / 32) * 32;
  const int ni = (nvec + threads - 1) / threads;
  switch (ni) {
    case 1: launch_pdl(rs_add_rmsnorm_ag_kernel<1>, dim3(a.ctas), dim3(threads), 0, stream, a); break;
    case 2: launch_pdl(rs_add_rmsnorm_ag_kernel<2>, dim3(a.ctas), dim3(threads), 0, stream, a); break;
    case 3: launch_pdl(rs_add_rmsnorm_ag_kernel<3>, dim3(a.ctas), dim3(threads), 0, stream, a); break;
    default: launch_pdl(rs_add_rmsnorm_ag_kernel<4>, dim3(a.ctas), dim3(threads), 0, stream, a); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_allreduce_oneshot(const CommArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  if (a.hidden % 8 || a.hidden > 8 * 256 * 4 || a.world > COMM_MAX_RANKS || a.ctas > COMM_MAX_CTAS || a.ctas < 1)
    return cudaErrorInvalidValue;
  const int nvec = a.hidden / 8;
  const int threads = nvec >= 256 ? 256 : ((nvec + 31) / 32) * 32;
  const int ni = (nvec + threads - 1) / threads;
  switch (ni) {
    case 1: launch_pdl(allreduce_oneshot_kernel<1>, dim3(a.ctas), dim3(threads), 0, stream, a); break;
    case 2: launch_pdl(allreduce_oneshot_kernel<2>, dim3(a.ctas), dim3(threads), 0, stream, a); break;
    case 3: launch_pdl(allreduce_oneshot_kernel<3>, dim3(a.ctas), dim3(threads), 0, stream, a); break;
    default: launch_pdl(allreduce_oneshot_kernel<4>, dim3(a.ctas), dim3(threads), 0, stream, a); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_allreduce_add_rmsnorm(const CommArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  if (a.hidden % 8 || a.hidden > 8 * 256 * 4 || a.world > COMM_MAX_RANKS || a.ctas > COMM_MAX_CTAS || a.ctas < 1)
    return cudaErrorInvalidValue;
  const int nvec = a.hidden / 8;
  const int threads = nvec >= 256 ? 256 : ((nvec + 31) / 32) * 32;
  const int ni = (nvec + threads - 1) / threads;
  switch (ni) {
    case 1: launch_pdl(allreduce_add_rmsnorm_kernel<1>, dim3(a.ctas), dim3(threads), 0, stream, a); break;
    case 2: launch_pdl(allreduce_add_rmsnorm_kernel<2>, dim3(a.ctas), dim3(threads), 0, stream, a); break;
    case 3: launch_pdl(allreduce_add_rmsnorm_kernel<3>, dim3(a.ctas), dim3(threads), 0, stream, a); break;
    default: launch_pdl(allreduce_add_rmsnorm_kernel<4>, dim3(a.ctas), dim3(threads), 0, stream, a); break;
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------------- KV block push
// Copy whole KV blocks of every (K/V, layer) plane from this GPU's pool into another
// GPU's pool (an IPC mapping) over NVLink: one launch per handoff, no staging buffer.
// Pools are [planes = 2 * layers][num_blocks][block_bytes]; CTA (i, plane) moves block
// src_ids[i] -> dst_ids[i] of that plane with 16-byte loads and stores.
__global__ void kv_push_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, const int* __restrict__ src_ids,
                               const int* __restrict__ dst_ids, int nb_src, int nb_dst, int64_t block_vec) {
  const int i = blockIdx.x, plane = blockIdx.y;
  const int s = src_ids[i], d = dst_ids[i];
  if (s < 0 || s >= nb_src || d < 0 || d >= nb_dst) {
    if (threadIdx.x == 0) atomicCAS(&g_comm_error, 0, 200);
    return;
  }
  const uint4* sp = src + ((int64_t)plane * nb_src + s) * block_vec;
  uint4* dp = dst + ((int64_t)plane * nb_dst + d) * block_vec;
  for (int64_t v = threadIdx.x; v < block_vec; v += blockDim.x) dp[v] = sp[v];
}

// Same copy for blocks whose size is a multiple of 4 bytes only (the per-block fp8 scales
// of a few KV heads): one 4-byte word per thread.
__global__ void kv_push_words_kernel(const uint32_t* __restrict__ src, uint32_t* __restrict__ dst,
                                     const int* __restrict__ src_ids, const int* __restrict__ dst_ids, int n, int planes,
                                     int nb_src, int nb_dst, int block_words) {
  const int64_t total = (int64_t)n * planes * block_words;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int w = (int)(t % block_words);
    const int64_t r = t / block_words;
    const int i = (int)(r % n), plane = (int)(r / n);
    const int s = src_ids[i], d = dst_ids[i];
    if (s < 0 || s >= nb_src || d < 0 || d >= nb_dst) {
      atomicCAS(&g_comm_error, 0, 201);
      continue;
    }
    dst[((int64_t)plane * nb_dst + d) * block_words + w] = src[((int64_t)plane * nb_src + s) * block_words + w];
  }
}

cudaError_t launch_kv_push(const void* src_pool, void* dst_pool, const int* src_ids, const int* dst_ids, int n,
                           int planes, int nb_src, int nb_dst, int64_t block_bytes, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  if (block_bytes % 16 == 0 && !((uintptr_t)src_pool & 15) && !((uintptr_t)dst_pool & 15)) {
    dim3 grid(n, planes);
    kv_push_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint4*>(src_pool), static_cast<uint4*>(dst_pool),
                                             src_ids, dst_ids, nb_src, nb_dst, block_bytes / 16);
    return cudaGetLastError();
  }
  if (block_bytes % 4 || ((uintptr_t)src_pool & 3) || ((uintptr_t)dst_pool & 3)) return cudaErrorInvalidValue;
  const int64_t total = (int64_t)n * planes * (block_bytes / 4);
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  kv_push_words_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint32_t*>(src_pool),
                                                   static_cast<uint32_t*>(dst_pool), src_ids, dst_ids, n, planes,
                                                   nb_src, nb_dst, (int)(block_bytes / 4));
  return cudaGetLastError();
}

// ------------------------------------------------------------ push completion flags
// The sender raises a 32-bit sequence number in a flag word that lives in the receiver's
// exported allocation once its push kernels (earlier in the same stream) have completed; the
// receiver's stream waits for that number before the pushed blocks are read.
__device__ int g_push_error = 0;

__global__ void push_signal_kernel(uint32_t* flag, uint32_t epoch) {
  // the push kernels before this one in the stream have completed; make their peer stores
  // visible system-wide before the flag
  fence_acq_rel_sys();
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(epoch) : "memory");
}

// status (optional): 1 when the flag arrived, 2 when the wait gave up
__global__ void push_wait_kernel(const uint32_t* flag, uint32_t epoch, uint64_t timeout_ns, int* status) {
  SpinBudget sb;
  for (;;) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (reached(v, epoch)) {
      if (status) *status = 1;
      return;
    }
    if (sb.expired(timeout_ns)) {
      atomicCAS(&g_push_error, 0, 210);  // the sender never signalled: the blocks are not usable
      if (status) *status = 2;
      return;
    }
    __nanosleep(256);
  }
}

cudaError_t launch_push_signal(uint32_t* flag, uint32_t epoch, cudaStream_t stream) {
  if (!flag || ((uintptr_t)flag & 3)) return cudaErrorInvalidValue;
  push_signal_kernel<<<1, 1, 0, stream>>>(flag, epoch);
  return cudaGetLastError();
}

cudaError_t launch_push_wait(const uint32_t* flag, uint32_t epoch, uint64_t timeout_ns, int* status,
                             cudaStream_t stream) {
  if (!flag || ((uintptr_t)flag & 3)) return cudaErrorInvalidValue;
  push_wait_kernel<<<1, 1, 0, stream>>>(flag, epoch, timeout_ns ? timeout_ns : COMM_WAIT_NS, status);
  return cudaGetLastError();
}

int push_error_code(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_push_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_push_error, &z, sizeof(int));
  }
  return v;
}

int comm_error_code(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_comm_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_comm_error, &z, sizeof(int));
  }
  return v;
}

// ----------------------------------------------------------- symmetric memory (IPC)
cudaError_t symm_alloc(size_t bytes, void** ptr, void* handle_out) {
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle_out), *ptr);
  if (e != cudaSuccess) cudaGetLastError();
  return e;
}

cudaError_t symm_open(const void* handle, void** ptr) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) cudaGetLastError();  // do not leave the error for the next launch check
  return e;
}

cudaError_t symm_close(void* peer_ptr) { return cudaIpcCloseMemHandle(peer_ptr); }

cudaError_t symm_free(void* ptr) { return cudaFree(ptr); }

}  // namespace nvb
