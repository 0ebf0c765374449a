// Allocation-free split-KV paged decode attention: the library's exported C interface.
//
// This entry point has no counterpart in the reference project; it is an addition of this
// library.  It serves callers that cannot call cudaMalloc: code running inside a captured CUDA
// graph whose memory pool is frozen, plug-ins hosted by an engine that owns every device
// allocation, and real-time loops in which an allocation may block.  The split-KV scratch lives
// in a fixed array in the library's device image instead (see attn_decode_noalloc.cu for the
// limits and the sharing rules).
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Decode attention over the paged KV pool, one query token per sequence.
//   q            [num_seqs, nq, 128] bf16 (row b at cu_seqlens_q[b])
//   k_cache      [num_blocks, nkv, block_size, 128] bf16, or fp8 e4m3 when kv_fp8 != 0
//   v_cache      same layout as k_cache
//   k_scale      [num_blocks, nkv] fp32 per-block per-head dequantisation scales (fp8 only, else NULL)
//   v_scale      same as k_scale
//   block_tables [num_seqs, block_table_width] int32 block ids
//   cu_seqlens_q [num_seqs + 1] int32; context_lens [num_seqs] int32 keys per sequence
//   out          [num_seqs, nq, 128] bf16, written by the call
// Requires head_dim == 128, nq % nkv == 0 with nq / nkv <= 16, a power-of-two block_size, and
// num_seqs * nq * splits <= nvb_attn_decode_noalloc_max_rows().  Returns a cudaError_t value:
// 0 on success, cudaErrorInvalidValue for arguments out of range (nothing is launched then).
// The first call on a device looks up the scratch array's device address, so make that call
// before any stream capture.  Calls whose kernels may overlap on the GPU race on the shared
// scratch: order them on one stream or with events.
int nvb_attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const float* k_scale,
                            const float* v_scale, const int* block_tables, int block_table_width,
                            const int* cu_seqlens_q, const int* context_lens, void* out, int num_seqs, int nq,
                            int nkv, int head_dim, int block_size, int num_blocks, int kv_fp8, int splits,
                            float softmax_scale, cudaStream_t stream);

// Largest num_seqs * nq * splits that one call of nvb_attn_decode_noalloc may use.
int nvb_attn_decode_noalloc_max_rows(void);

#ifdef __cplusplus
}
#endif
