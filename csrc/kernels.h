// Host-side launch entry points of the sm_100a kernels (raw pointers, no torch types).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace nvb {

// src_rows: rows of x (and residual_in) that row_index may address (checked, see NVB_BOUNDS_CHECK).
cudaError_t launch_add_rmsnorm(const void* x, int64_t x_stride, const void* residual_in, void* residual_out,
                               const void* w, void* out, int rows, int H, float eps, const int* row_index,
                               cudaStream_t stream, int src_rows = 0x7fffffff);
int norm_check_code(int reset);
int bounds_check_enabled();
int qkv_check_code(int reset);
cudaError_t launch_silu_mul(const void* x, void* out, int T, int I, cudaStream_t stream);
cudaError_t launch_embedding(const int* ids, const void* table, int rows, int vocab_start, void* out, int T, int H,
                             cudaStream_t stream);
cudaError_t launch_qkv_post(const void* qkv, int64_t qkv_stride, void* q_out, const void* q_norm, const void* k_norm,
                            float eps, const int* positions, const float* cos_sin, void* k_cache, void* v_cache,
                            float* k_scale, float* v_scale, const int* slots, int T, int nq, int nkv, int head_dim,
                            int block_size, int kv_fp8, cudaStream_t stream, int num_blocks = 0x7fffffff);

struct AttnLaunch {
  const void* q;
  const void* k_cache;
  const void* v_cache;
  const float* k_scale;
  const float* v_scale;
  const int* block_tables;
  int W;
  const int* cu_q;
  const int* ctx_lens;
  void* out;
  float* part_o;
  float* part_lse;
  int nq, nkv, head_dim, block_size, num_blocks;
  int splits;
  int seq_offset;
  int num_seqs;
  int kv_fp8;
  float softmax_scale;
};

int attn_decode_splits(int num_seqs, int nkv, int max_ctx, int num_sms);
cudaError_t launch_attn_decode(const AttnLaunch& L, cudaStream_t stream);
cudaError_t launch_attn_prefill(const AttnLaunch& L, int max_q_len, cudaStream_t stream);
// total_q: rows of q (tokens of the whole launch's q tensor, for its tensor map; <= 0 forces the
// mma.sync kernel); use_tc: 1 = tcgen05 kernel where it applies (bf16 KV), 0 = mma.sync kernel.
cudaError_t launch_attn_prefill_ex(const AttnLaunch& L, int max_q_len, int total_q, int use_tc, cudaStream_t stream);
// Error word set by an attention kernel that gave up on a bounded wait (0 = none).
int attn_error_code(int reset);

int sample_num_chunks(int rows, int V);
cudaError_t launch_sample(const void* logits, int logits_is_bf16, int64_t ld, int rows, int V, int64_t col_offset,
                          const float* temps, const int64_t* seed_step, float* part_val, int* part_idx, int nchunk,
                          int* out_tok, float* out_val, cudaStream_t stream);

// Row-parallel sampler (one CTA per row): greedy / temperature / top-p over a vocabulary
// shard, with the cross-rank combination inside the kernel when world > 1 (see sampling.cu).
constexpr int SAMPLE_NB = 1024;  // histogram bins per level of the top-p threshold search
struct SampleX {
  int world = 1, rank = 0, rows_cap = 0;
  float* x[8] = {};        // every rank's exchange area (floats; regions of rounds 1-4)
  uint32_t* f[8] = {};     // every rank's flag words [4 rounds][rows_cap][world]
  uint32_t* ctrl = nullptr;  // this rank's [0] completed calls, [1] finished CTAs
  uint64_t timeout_ns = 10000000000ull;
};
// Floats of one rank's exchange area / words of its flag area for `rows_cap` rows.
inline int64_t sample_x_floats(int world, int rows_cap) {
  const int64_t wr = (int64_t)world * rows_cap;
  return wr + wr * (SAMPLE_NB + 1) + wr * SAMPLE_NB + wr * 2;
}
inline int64_t sample_f_words(int world, int rows_cap) { return 4LL * rows_cap * world + 2; }
int sample_rows_capacity();
cudaError_t launch_sample_rows(const void* logits, int logits_is_bf16, int64_t ld, int rows, int V, int64_t col_offset,
                               const float* temps, const float* top_p, const int64_t* seed_step, int* out_tok,
                               float* out_val, const SampleX& X, cudaStream_t stream);
int sample_error_code(int reset);
// Tokens (and, optionally, winning scores) from the per-row keys of the lm_head GEMM's sampling
// epilogue; zeroes the keys for the next launch.
cudaError_t launch_sample_keys(unsigned long long* keys, int rows, int* out_tok, float* out_val, cudaStream_t stream);

}  // namespace nvb
