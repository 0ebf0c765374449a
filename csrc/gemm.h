// tcgen05 GEMM host interface.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace nvb {

struct GemmPlan {
  int swap;          // 1: weights fill the 128-row MMA side (decode); 0: tokens do (prefill)
  int bn;            // tile width along the other operand (32/64/128/256)
  int tiles_p, tiles_q;
  int num_kb, kb_per_split, splits;
  int grid;
  int64_t ws_ld;     // split-K scratch row length (fp32 elements)
  int64_t ws_elems;  // split-K scratch size needed (fp32 elements), 0 if none
  int tiles;         // output tiles
  int prefetch_w;    // stream the weights through an L2 prefetch lookahead
};

// Plan C[m, n] = X[m, k] * W[n, k]^T.  force_* < 0 / 0 = automatic.
GemmPlan gemm_plan(int m, int n, int k, int force_swap, int force_bn, int force_splits);

// ws: fp32 split-K scratch (plan.ws_elems); counters: 4 int32 per output tile, all zero
// before the first launch (the kernel leaves them zero).
cudaError_t gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int m, int n, int k,
                      const GemmPlan& plan, float* ws, int* counters, cudaStream_t stream);

// Same product, configuration chosen by timing candidates on first use of a shape (outside
// stream capture) and cached; inside a capture the cached or heuristic plan is used.
cudaError_t gemm_bf16_tuned(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int m, int n,
                            int k, cudaStream_t stream, GemmPlan* chosen);

// Error word written by a GEMM that gave up on a bounded wait (0 = none).
int gemm_error_code(int reset);

}  // namespace nvb
