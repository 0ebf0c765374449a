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
// COMM_CTRL_WORDS local control words: [0] calls completed, [1] go, [2] CTAs done, [3] go
// error, [4] CTAs done of a reduce-scatter GEMM; then the reduce-scatter flags: RS slot p =
// "rank p's GEMM has stored its partial rows for call n here", AG slot p = "rank p has
// stored its normalised rows of call n here".
constexpr int COMM_CTRL_WORDS = 8;
constexpr size_t COMM_ONESHOT_FLAGS = 0;                      // word offsets
constexpr size_t COMM_TWOSHOT_A = COMM_MAX_RANKS;
constexpr size_t COMM_TWOSHOT_B = 2 * COMM_MAX_RANKS;
constexpr size_t COMM_CTRL = 3 * COMM_MAX_RANKS;
constexpr size_t COMM_CTRL_GEMM_DONE = COMM_CTRL + 4;
constexpr size_t COMM_RS_FLAGS = COMM_CTRL + COMM_CTRL_WORDS;
constexpr size_t COMM_AG_FLAGS = COMM_RS_FLAGS + COMM_MAX_RANKS;
constexpr size_t COMM_FLAG_BYTES = 256;
static_assert((COMM_AG_FLAGS + COMM_MAX_RANKS) * sizeof(uint32_t) <= COMM_FLAG_BYTES, "flag region");
// Rows of one reduce-scatter receive slot (the decode GEMM's row limit).
constexpr int COMM_RS_MAX_ROWS = 256;

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

// Owner side of the GEMM -> reduce-scatter path.  Rank r owns rows [r rs_rows, (r+1) rs_rows)
// of the step's `rows` tokens.  Every rank's reduce-scatter GEMM has stored its partial sums of
// those rows in rs[p][i][H] (slot p = source rank) and raised RS flag p.  The kernel waits for
// the world flags, sums the partials, adds the residual (owned rows of `res`, kept only here),
// applies RMSNorm and stores the normalised rows into every rank's OUT (all-gather by peer
// stores); the last CTA then raises this rank's AG flag at every rank and waits for every
// rank's, so when the kernel completes every rank's OUT holds all rows.
struct RsNormArgs {
  const __nv_bfloat16* rs;              // this rank's receive area [world][COMM_RS_MAX_ROWS][hidden]
  __nv_bfloat16* res;                   // this rank's residual rows [rows][hidden] (owned rows used)
  __nv_bfloat16* out[COMM_MAX_RANKS];   // every rank's OUT [rows][hidden]
  uint32_t* flags[COMM_MAX_RANKS];      // every rank's FLAGS region
  const __nv_bfloat16* weight;
  int rank, world, rows, rs_rows, hidden, ctas, has_residual;
  uint64_t timeout_ns;
  float eps;
};
cudaError_t launch_rs_add_rmsnorm_ag(const RsNormArgs& a, cudaStream_t stream);
// Single-barrier variant: every rank reduces every row (small batches; IN must rotate).
cudaError_t launch_allreduce_oneshot(const CommArgs& a, cudaStream_t stream);
int comm_error_code(int reset);

// Copy blocks src_ids[i] -> dst_ids[i] of every plane of [planes][nb][block_bytes] pools.
cudaError_t launch_kv_push(const void* src_pool, void* dst_pool, const int* src_ids, const int* dst_ids, int n,
                           int planes, int nb_src, int nb_dst, int64_t block_bytes, cudaStream_t stream);

// Push completion: after the pushes of one handoff, raise `flag` (a word of the receiver's
// exported allocation) to `epoch`; the receiver's stream waits (bounded; error word 210 on
// expiry, read with push_error_code) until the flag has reached `epoch`.
constexpr int PUSH_FLAG_SLOTS = 256;  // one word per sending worker
cudaError_t launch_push_signal(uint32_t* flag, uint32_t epoch, cudaStream_t stream);
cudaError_t launch_push_wait(const uint32_t* flag, uint32_t epoch, uint64_t timeout_ns, int* status,
                             cudaStream_t stream);
int push_error_code(int reset);

cudaError_t symm_alloc(size_t bytes, void** ptr, void* handle_out);  // handle_out: 64 bytes
cudaError_t symm_open(const void* handle, void** ptr);
cudaError_t symm_close(void* peer_ptr);
cudaError_t symm_free(void* ptr);

}  // namespace nvb
