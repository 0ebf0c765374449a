// Tensor-parallel fused all-reduce over NVLink peer memory: host interface.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <cuda_bf16.h>

namespace nvb {

constexpr int COMM_MAX_RANKS = 8;
constexpr int COMM_MAX_CTAS = 256;
// FLAGS region (uint32 words): [3 barriers][COMM_MAX_RANKS] cross-rank flags (one-shot,
// two-shot phase A, two-shot phase B; slot p holds rank p's latest call number), then
// COMM_CTRL_WORDS local control words: [0] calls completed, [1] go, [2] CTAs done.
constexpr int COMM_CTRL_WORDS = 8;
constexpr size_t COMM_ONESHOT_FLAGS = 0;                      // word offsets
constexpr size_t COMM_TWOSHOT_A = COMM_MAX_RANKS;
constexpr size_t COMM_TWOSHOT_B = 2 * COMM_MAX_RANKS;
constexpr size_t COMM_CTRL = 3 * COMM_MAX_RANKS;
constexpr size_t COMM_FLAG_BYTES = 256;
static_assert((COMM_CTRL + COMM_CTRL_WORDS) * sizeof(uint32_t) <= COMM_FLAG_BYTES, "flag region");

struct CommArgs {
  __nv_bfloat16* in[COMM_MAX_RANKS];   // every rank's IN buffer (peer pointers)
  __nv_bfloat16* res[COMM_MAX_RANKS];
  __nv_bfloat16* out[COMM_MAX_RANKS];
  uint32_t* flags[COMM_MAX_RANKS];
  const __nv_bfloat16* weight;
  int rank, world, rows, hidden, ctas, has_residual;
  uint64_t timeout_ns;                 // bound of every peer wait (0: the default, 10 s)
  float eps;
};

cudaError_t launch_allreduce_add_rmsnorm(const CommArgs& a, cudaStream_t stream);
// Single-barrier variant: every rank reduces every row (small batches; IN must rotate).
cudaError_t launch_allreduce_oneshot(const CommArgs& a, cudaStream_t stream);
int comm_error_code(int reset);

// Copy blocks src_ids[i] -> dst_ids[i] of every plane of [planes][nb][block_bytes] pools.
cudaError_t launch_kv_push(const void* src_pool, void* dst_pool, const int* src_ids, const int* dst_ids, int n,
                           int planes, int nb_src, int nb_dst, int64_t block_bytes, cudaStream_t stream);

cudaError_t symm_alloc(size_t bytes, void** ptr, void* handle_out);  // handle_out: 64 bytes
cudaError_t symm_open(const void* handle, void** ptr);
cudaError_t symm_close(void* peer_ptr);
cudaError_t symm_free(void* ptr);

}  // namespace nvb
