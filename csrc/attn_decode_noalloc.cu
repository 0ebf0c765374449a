// Split-KV paged decode attention for callers that cannot allocate device memory.
//
// This entry point has no counterpart in the reference project; it is an addition of
// this library.  Some callers cannot call cudaMalloc: code that runs inside a captured
// CUDA graph whose memory pool is frozen, plug-ins hosted by an engine that owns every
// allocation, or real-time loops where an allocation may block.  The regular decode
// attention (launch_attn_decode) needs scratch memory for the per-split partial outputs
// whenever a sequence's context is split across CTAs, and its Python wrapper allocates
// that scratch through torch.  nvb_attn_decode_noalloc runs the same kernels with the
// scratch taken from a fixed array that lives in this library's device image instead:
//
//   * the scratch is the file-scope array g_noalloc_scratch below: NOALLOC_MAX_ROWS
//     rows of (128 partial-output floats + 1 log-sum-exp float), about 4.2 MB.  Every
//     GPU that loads this library holds that array until the process exits;
//   * a call needs num_seqs * nq * splits rows; larger requests are rejected with
//     cudaErrorInvalidValue before anything is launched (lower `splits`, or split the
//     batch into several calls);
//   * nothing in the scratch has to start at zero.  Every row of the partial log-sum-exps a
//     call reads is written by that call; a split that gets no keys writes only its
//     log-sum-exp (-inf), and the combine step skips such splits without reading their
//     partial-output rows, so stale contents from an earlier call (NaN included) never
//     reach the output;
//   * all calls share the one array per device.  Two calls whose kernels may overlap on
//     the GPU (different streams without ordering between them) race on it; order them
//     on one stream, or with events;
//   * the device address of the array is obtained with cudaGetSymbolAddress the first
//     time a device is used (host code only sees a host-side stand-in for the symbol).
//     That first call per device should therefore happen before any stream capture;
//   * no cudaMalloc, cudaFree or allocating library routine is called.
//
// The C declarations are in attn_decode_noalloc.h.  Inputs are the same as
// launch_attn_decode's (kernels.h); the caller passes the output buffer.  Returns a
// cudaError_t value (0 on success).
#include <mutex>

#include "attn_decode_noalloc.h"
#include "common.cuh"
#include "kernels.h"

namespace {

constexpr int NOALLOC_HEAD_DIM = 128;
constexpr int NOALLOC_MAX_ROWS = 8192;  // (sequence, query head, split) rows
constexpr int NOALLOC_MAX_DEVICES = 64;

// [NOALLOC_MAX_ROWS * 128 partial outputs][NOALLOC_MAX_ROWS log-sum-exps], fp32.
static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_MAX_ROWS * (NOALLOC_HEAD_DIM + 1)];

std::mutex g_mu;
float* g_dev_ptr[NOALLOC_MAX_DEVICES] = {};

// Device address of the scratch array on the current device (set up once per device).
cudaError_t scratch_ptr(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_dev_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_dev_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_dev_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int nvb_attn_decode_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const float* k_scale, const float* v_scale,
    const int* block_tables, int block_table_width, const int* cu_seqlens_q, const int* context_lens, void* out,
    int num_seqs, int nq, int nkv, int head_dim, int block_size, int num_blocks, int kv_fp8, int splits,
    float softmax_scale, cudaStream_t stream) {
  if (num_seqs <= 0) return (int)cudaSuccess;
  if (head_dim != NOALLOC_HEAD_DIM || splits < 1) return (int)cudaErrorInvalidValue;
  // checked here, before any division by nkv or launch
  if (nq <= 0 || nkv <= 0 || nq % nkv || nq / nkv > 16) return (int)cudaErrorInvalidValue;
  if (block_size <= 0 || (block_size & (block_size - 1)) || num_blocks <= 0 || block_table_width <= 0)
    return (int)cudaErrorInvalidValue;
  if (!q || !k_cache || !v_cache || !block_tables || !cu_seqlens_q || !context_lens || !out)
    return (int)cudaErrorInvalidValue;
  if (kv_fp8 && (!k_scale || !v_scale)) return (int)cudaErrorInvalidValue;
  if ((long long)num_seqs * nq * splits > NOALLOC_MAX_ROWS) return (int)cudaErrorInvalidValue;
  float* scratch = nullptr;
  cudaError_t e = scratch_ptr(&scratch);
  if (e != cudaSuccess) return (int)e;
  nvb::AttnLaunch L{};
  L.q = q;
  L.k_cache = k_cache;
  L.v_cache = v_cache;
  L.k_scale = k_scale;
  L.v_scale = v_scale;
  L.block_tables = block_tables;
  L.W = block_table_width;
  L.cu_q = cu_seqlens_q;
  L.ctx_lens = context_lens;
  L.out = out;
  L.part_o = scratch;
  L.part_lse = scratch + (size_t)NOALLOC_MAX_ROWS * NOALLOC_HEAD_DIM;
  L.nq = nq;
  L.nkv = nkv;
  L.head_dim = head_dim;
  L.block_size = block_size;
  L.num_blocks = num_blocks;
  L.splits = splits;
  L.seq_offset = 0;
  L.num_seqs = num_seqs;
  L.kv_fp8 = kv_fp8;
  L.softmax_scale = softmax_scale;
  return (int)nvb::launch_attn_decode(L, stream);
}

// Largest num_seqs * nq * splits one call may use.
extern "C" __attribute__((visibility("default"))) int nvb_attn_decode_noalloc_max_rows(void) { return NOALLOC_MAX_ROWS; }
