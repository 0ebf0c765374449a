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
  int streamk;       // 1: stream-K (even split of tiles x k-blocks over the grid; needs ws + counters)
  int mt;            // 128-row sub-tiles of the token operand per output tile (1 or 2)
  int dec;           // 1: decode kernel (all m <= 256 tokens per CTA, runtime bn, cluster split-K);
                     // 2: skinny kernel (weights on the MMA's M side, mt = tokens per tile,
                     //    bn = weight rows per CTA, cluster split-K);
                     // 3: CTA-pair kernel (128 < m <= 256 tokens, M = 256 over two CTAs,
                     //    bn = weight rows per pair, tiles = pairs)
  int stages, smem;  // decode kernel: weight-ring depth and dynamic shared memory
  int a_stages;      // decode kernel: activation-ring depth
};

// Plan C[m, n] = X[m, k] * W[n, k]^T.  force_swap < 0 / force_bn 0 / force_splits 0 =
// automatic; force_splits = -1 or -2 selects stream-K with 1 or 2 sub-tiles of 128 tokens.
GemmPlan gemm_plan(int m, int n, int k, int force_swap, int force_bn, int force_splits);

// The rank-th cheapest decode-kernel configuration for C[m, n] (m <= 256) by the cost
// model; false if there is none.
bool gemm_dec_plan(int m, int n, int k, int rank, GemmPlan* plan);

// The rank-th skinny-kernel configuration (fewest bytes per CTA first) for C[m, n], m <= 256;
// false if there is none.
bool gemm_skinny_plan(int m, int n, int k, int rank, int act, GemmPlan* plan);
// Skinny kernel with W in the blocked layout [n / 128][k / 64][128][64] (blocked = 1) or row-major.
// trace (optional): 328 uint64 %globaltimer stamps per CTA (see SkParams).
cudaError_t gemm_skinny_run(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int m, int n,
                            int k, const GemmPlan& plan, int act, int blocked, cudaStream_t stream,
                            uint64_t* trace = nullptr);

// The rank-th CTA-pair kernel configuration (fewest bytes per CTA first) for C[m, n],
// 128 < m <= 256; false if there is none.  Run it with gemm_bf16.
bool gemm_pair_plan(int m, int n, int k, int rank, int act, GemmPlan* plan);

// Decode kernel with an explicit (bn, splits, activation-ring depth) configuration.
cudaError_t gemm_dec_explicit(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int m,
                              int n, int k, int bn, int splits, int a_stages, cudaStream_t stream);

// Sampling epilogue of the lm_head GEMM: the product is not stored; each output value is rounded
// to bf16, noised (Gumbel-max, for rows whose temperature is > 0) and folded into a per-token key
// by an atomic max, so that the key of token row i names the sampled column.  keys[m] must be zero
// before the launch (sample_keys decodes the keys and zeroes them again).
struct GemmSampleEpilogue {
  unsigned long long* keys = nullptr;  // [m]
  const float* temps = nullptr;        // [m] temperature per row (<= 0: greedy)
  const int64_t* seed_step = nullptr;  // (seed, step) of the noise
  int64_t col_offset = 0;              // global column of output feature 0 (vocab shard start)
};

// ws: fp32 split-K scratch (plan.ws_elems); counters: 4 int32 per output tile, all zero
// before the first launch (the kernel leaves them zero).
// act = 1: fused SiLU-and-mul epilogue.  W's rows are gate/up interleaved in groups of 16
// (rows 32j..32j+15 gate features 16j..16j+15, rows 32j+16..32j+31 the matching up
// features) and C receives silu(gate) * up: [m, n / 2] with row stride ldc.  Needs n % 32
// == 0, the normal orientation and a tile width that is a multiple of 32.
// se (optional): the sampling epilogue instead of storing C (persistent-kernel plans only:
// sample_plan_ok).
cudaError_t gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int m, int n, int k,
                      const GemmPlan& plan, float* ws, int* counters, cudaStream_t stream, int act = 0,
                      const GemmSampleEpilogue* se = nullptr);
bool sample_plan_ok(const GemmPlan& plan);

// lm_head GEMM with the sampling epilogue.  The plan is chosen on first use of a shape by timing the
// persistent-kernel candidates with the epilogue itself (tune = true, outside stream capture), then
// cached; inside a capture, or without tuning, the heuristic plan is used.
cudaError_t gemm_bf16_sample(const void* x, int64_t ldx, const void* w, int64_t ldw, int m, int n, int k,
                             const GemmSampleEpilogue& se, float* ws, int64_t ws_elems, int* counters,
                             int64_t num_counters, bool tune, cudaStream_t stream, GemmPlan* chosen);

// Same product, configuration chosen by timing candidates on first use of a shape (outside
// stream capture) and cached; inside a capture the cached or heuristic plan is used.
// ws / ws_elems / counters / num_counters: scratch for stream-K candidates (may be null).
cudaError_t gemm_bf16_tuned(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int m, int n,
                            int k, float* ws, int64_t ws_elems, int* counters, int64_t num_counters,
                            cudaStream_t stream, GemmPlan* chosen, int act = 0);

// Reduce-scatter epilogue of the decode GEMM (tensor parallelism): instead of writing C
// locally, output row i is stored straight into the memory of the rank that owns it, rank
// i / rows, at dst[owner] + (i % rows) * ldc (that rank's receive slot for this rank; a peer
// pointer for every rank but this one).  When every CTA has stored its rows, the last CTA to
// finish raises this rank's arrival word at every rank: *flag[r] = *calls + 1, the number of
// the reduction this GEMM feeds.  *ctas_done counts the finished CTAs and is zero between
// launches (the last CTA resets it).
struct GemmRsEpilogue {
  int rows = 0;          // output rows per owner rank (0: plain local output)
  int world = 0;
  void* dst[8] = {};     // bf16 [rows][ldc] receive slot per owner rank
  uint32_t* flag[8] = {};
  const uint32_t* calls = nullptr;
  uint32_t* ctas_done = nullptr;
};

// C[m, n] = X W^T with the reduce-scatter epilogue (decode kernel, m <= 256, k % 64 == 0).
// The configuration is chosen on first use of a shape by timing the decode-kernel candidates
// with a plain local output into tune_c[m, n] (row stride tune_ldc; outside stream capture),
// then cached.  Returns cudaErrorNotSupported for shapes the decode kernel cannot run.
cudaError_t gemm_bf16_rs(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t ldc, int m, int n, int k,
                         const GemmRsEpilogue& rs, void* tune_c, int64_t tune_ldc, cudaStream_t stream,
                         GemmPlan* chosen);

// Deterministic mode (default: environment NVB_DETERMINISTIC): plans chosen from the shape alone,
// never by timing, so every process runs a shape with the same kernel and split-K order.
void gemm_set_deterministic(int on);
int gemm_deterministic();

// Error word written by a GEMM that gave up on a bounded wait (0 = none).
int gemm_error_code(int reset);

}  // namespace nvb
