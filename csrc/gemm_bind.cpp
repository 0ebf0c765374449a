// Python bindings of the tcgen05 GEMM.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "comm.h"
#include "gemm.h"
#include "kernels.h"

namespace {

// out[m, n] = x[m, k] @ w[n, k]^T   (bf16 in/out, fp32 accumulation)
void linear(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, const c10::optional<at::Tensor>& ws,
            const c10::optional<at::Tensor>& counters, int64_t force_swap, int64_t force_bn, int64_t force_splits,
            int64_t act) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16, "bf16 required");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2, "2-D tensors required");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "unit inner stride required");
  const int m = (int)x.size(0), k = (int)x.size(1), n = (int)w.size(0);
  TORCH_CHECK(w.size(1) == k && out.size(0) == m && out.size(1) == (act ? n / 2 : n), "shape mismatch");
  auto pl = nvb::gemm_plan(m, n, k, (int)force_swap, (int)force_bn, (int)force_splits);
  float* wsp = nullptr;
  int* ctr = nullptr;
  if (pl.ws_elems > 0) {
    TORCH_CHECK(ws.has_value() && ws->scalar_type() == at::kFloat && ws->numel() >= pl.ws_elems,
                "split-K scratch too small: need ", pl.ws_elems, " fp32 elements");
    TORCH_CHECK(counters.has_value() && counters->scalar_type() == at::kInt && counters->numel() >= 4 * pl.tiles,
                "split-K counters too small: need ", 4 * pl.tiles);
    wsp = ws->data_ptr<float>();
    ctr = counters->data_ptr<int>();
  }
  at::cuda::CUDAGuard g(x.device());
  cudaError_t e = nvb::gemm_bf16(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(), out.stride(0),
                                 m, n, k, pl, wsp, ctr, at::cuda::getCurrentCUDAStream().stream(), (int)act);
  TORCH_CHECK(e == cudaSuccess, "gemm_bf16 failed: ", cudaGetErrorString(e));
}

// Autotuned entry point used by the model (see gemm_bf16_tuned).
std::vector<int64_t> linear_tuned(const at::Tensor& x, const at::Tensor& w, at::Tensor& out,
                                  const c10::optional<at::Tensor>& ws, const c10::optional<at::Tensor>& counters,
                                  int64_t act) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16, "bf16 required");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2, "2-D tensors required");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "unit inner stride required");
  const int m = (int)x.size(0), k = (int)x.size(1), n = (int)w.size(0);
  TORCH_CHECK(w.size(1) == k && out.size(0) == m && out.size(1) == (act ? n / 2 : n), "shape mismatch");
  at::cuda::CUDAGuard g(x.device());
  float* wsp = nullptr;
  int* ctr = nullptr;
  int64_t ws_n = 0, ctr_n = 0;
  if (ws.has_value() && counters.has_value()) {
    TORCH_CHECK(ws->scalar_type() == at::kFloat && counters->scalar_type() == at::kInt, "fp32 ws, int32 counters");
    wsp = ws->data_ptr<float>();
    ws_n = ws->numel();
    ctr = counters->data_ptr<int>();
    ctr_n = counters->numel();
  }
  nvb::GemmPlan pl{};
  cudaError_t e = nvb::gemm_bf16_tuned(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(),
                                       out.stride(0), m, n, k, wsp, ws_n, ctr, ctr_n,
                                       at::cuda::getCurrentCUDAStream().stream(), &pl, (int)act);
  TORCH_CHECK(e == cudaSuccess, "gemm_bf16 failed: ", cudaGetErrorString(e));
  // (swap, bn, tiles_p, tiles_q, splits, grid); splits < 0: stream-K with -splits sub-tiles;
  // splits >= 100: decode kernel with splits - 100 K slices; >= 200: skinny kernel with
  // splits - 200 K slices (bn = weight rows per CTA)
  return {pl.swap, pl.bn, pl.tiles_p, pl.tiles_q,
          pl.dec == 3 ? 300 : pl.dec == 2 ? 200 + pl.splits : pl.dec ? 100 + pl.splits : pl.streamk ? -pl.mt : pl.splits, pl.grid};
}

// lm_head GEMM with the sampler in its epilogue: tok[i] = the token sampled from row i of x @ w^T
// (greedy where temps[i] <= 0, else Gumbel-max at temps[i]), the logits never stored.  keys:
// int64 [>= m] scratch, zero between calls.  force_* (any set): an explicit persistent-kernel plan
// (as `linear`); otherwise the tuned one (tune: time candidates on first use of the shape).
std::vector<int64_t> linear_sample(const at::Tensor& x, const at::Tensor& w, at::Tensor& keys, const at::Tensor& temps,
                                   const at::Tensor& seed_step, int64_t col_offset, at::Tensor& out_tok,
                                   const c10::optional<at::Tensor>& out_val, const c10::optional<at::Tensor>& ws,
                                   const c10::optional<at::Tensor>& counters, bool tune, int64_t force_swap,
                                   int64_t force_bn, int64_t force_splits) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && keys.is_cuda(), "CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "bf16 required");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1, "2-D, unit inner stride");
  const int m = (int)x.size(0), k = (int)x.size(1), n = (int)w.size(0);
  TORCH_CHECK(w.size(1) == k, "shape mismatch");
  TORCH_CHECK(keys.scalar_type() == at::kLong && keys.is_contiguous() && keys.numel() >= m, "keys int64 [>= m]");
  TORCH_CHECK(temps.scalar_type() == at::kFloat && temps.numel() >= m, "temps fp32 [>= m]");
  TORCH_CHECK(seed_step.scalar_type() == at::kLong && seed_step.numel() >= 2, "seed_step int64[2]");
  TORCH_CHECK(out_tok.scalar_type() == at::kInt && out_tok.numel() >= m, "out_tok int32 [>= m]");
  at::cuda::CUDAGuard g(x.device());
  float* wsp = nullptr;
  int* ctr = nullptr;
  int64_t ws_n = 0, ctr_n = 0;
  if (ws.has_value() && counters.has_value()) {
    TORCH_CHECK(ws->scalar_type() == at::kFloat && counters->scalar_type() == at::kInt, "fp32 ws, int32 counters");
    wsp = ws->data_ptr<float>();
    ws_n = ws->numel();
    ctr = counters->data_ptr<int>();
    ctr_n = counters->numel();
  }
  nvb::GemmSampleEpilogue se;
  se.keys = reinterpret_cast<unsigned long long*>(keys.data_ptr<int64_t>());
  se.temps = temps.data_ptr<float>();
  se.seed_step = seed_step.data_ptr<int64_t>();
  se.col_offset = col_offset;
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  nvb::GemmPlan pl{};
  cudaError_t e;
  if (force_swap >= 0 || force_bn > 0 || force_splits != 0) {
    pl = nvb::gemm_plan(m, n, k, (int)force_swap, (int)force_bn, (int)force_splits);
    TORCH_CHECK(nvb::sample_plan_ok(pl), "the sampling epilogue needs a persistent-kernel plan");
    TORCH_CHECK(!pl.streamk || (wsp && pl.ws_elems <= ws_n && 4 * (int64_t)pl.tiles <= ctr_n),
                "stream-K scratch too small");
    e = nvb::gemm_bf16(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), nullptr, 0, m, n, k, pl, wsp, ctr, stream,
                       0, &se);
  } else {
    e = nvb::gemm_bf16_sample(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), m, n, k, se, wsp, ws_n, ctr, ctr_n,
                              tune, stream, &pl);
  }
  TORCH_CHECK(e == cudaSuccess, "gemm_bf16 (sampling epilogue) failed: ", cudaGetErrorString(e));
  e = nvb::launch_sample_keys(se.keys, m, out_tok.data_ptr<int>(),
                              out_val.has_value() ? out_val->data_ptr<float>() : nullptr, stream);
  TORCH_CHECK(e == cudaSuccess, "sample_keys failed: ", cudaGetErrorString(e));
  return {pl.swap, pl.bn, pl.tiles_p, pl.tiles_q, pl.streamk ? -pl.mt : pl.splits, pl.grid};
}

std::vector<int64_t> plan(int64_t m, int64_t n, int64_t k, int64_t force_swap, int64_t force_bn,
                          int64_t force_splits) {
  auto pl = nvb::gemm_plan((int)m, (int)n, (int)k, (int)force_swap, (int)force_bn, (int)force_splits);
  return {pl.swap, pl.bn, pl.tiles_p, pl.tiles_q, pl.splits, pl.grid, pl.ws_elems, 4 * (int64_t)pl.tiles};
}

// Decode kernel with the rank-th cheapest configuration of the cost model; returns
// (mt, bn, splits, weight stages, activation stages), empty if there is no such configuration.
std::vector<int64_t> linear_dec(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, int64_t rank,
                                int64_t act) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16, "bf16 required");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "unit inner stride required");
  const int m = (int)x.size(0), k = (int)x.size(1), n = (int)w.size(0);
  TORCH_CHECK(w.size(1) == k && out.size(0) == m && out.size(1) == (act ? n / 2 : n), "shape mismatch");
  nvb::GemmPlan pl{};
  if (!nvb::gemm_dec_plan(m, n, k, (int)rank, &pl)) return {};
  if (act && pl.bn % 32) return {0};
  at::cuda::CUDAGuard g(x.device());
  cudaError_t e = nvb::gemm_bf16(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(), out.stride(0),
                                 m, n, k, pl, nullptr, nullptr, at::cuda::getCurrentCUDAStream().stream(), (int)act);
  TORCH_CHECK(e == cudaSuccess, "gemm_bf16 failed: ", cudaGetErrorString(e));
  return {pl.mt, pl.bn, pl.splits, pl.stages, pl.a_stages};
}

// Decode kernel with an explicit (bn, splits, activation-ring depth) configuration.
void linear_dec_cfg(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, int64_t bn, int64_t splits,
                    int64_t a_stages) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16, "bf16 required");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "unit inner stride required");
  const int m = (int)x.size(0), k = (int)x.size(1), n = (int)w.size(0);
  TORCH_CHECK(w.size(1) == k && out.size(0) == m && out.size(1) == n, "shape mismatch");
  at::cuda::CUDAGuard g(x.device());
  cudaError_t e = nvb::gemm_dec_explicit(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(),
                                         out.stride(0), m, n, k, (int)bn, (int)splits, (int)a_stages,
                                         at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(e == cudaSuccess, "gemm_dec_explicit failed: ", cudaGetErrorString(e));
}

// Row-parallel GEMM with the reduce-scatter epilogue (tensor parallelism): x @ w^T whose row i
// is stored into rank i / rs_rows's symmetric receive area (slot `rank`) instead of locally;
// bases[p] = rank p's symmetric buffer, rs_off / flag_off = byte offsets of the receive area
// and the flag words in it.  tune_out [m, n] receives the plain output of the candidates timed
// on the first use of a shape.  Returns (mt, bn, splits) of the decode-kernel plan used.
std::vector<int64_t> linear_rs(const at::Tensor& x, const at::Tensor& w, std::vector<int64_t> bases, int64_t rs_off,
                               int64_t flag_off, int64_t rank, int64_t rs_rows, at::Tensor& tune_out) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && tune_out.is_cuda(), "CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  tune_out.scalar_type() == at::kBFloat16, "bf16 required");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 && tune_out.stride(1) == 1,
              "2-D tensors with unit inner stride required");
  const int m = (int)x.size(0), k = (int)x.size(1), n = (int)w.size(0);
  const int world = (int)bases.size();
  TORCH_CHECK(w.size(1) == k && tune_out.size(0) >= m && tune_out.size(1) == n, "shape mismatch");
  TORCH_CHECK(world >= 1 && world <= nvb::COMM_MAX_RANKS && rank >= 0 && rank < world, "bad rank / world");
  TORCH_CHECK(rs_rows >= 1 && rs_rows <= nvb::COMM_RS_MAX_ROWS && (int64_t)rs_rows * world >= m, "bad rs_rows");
  nvb::GemmRsEpilogue rs;
  rs.rows = (int)rs_rows;
  rs.world = world;
  const int64_t slot_bytes = (int64_t)nvb::COMM_RS_MAX_ROWS * n * 2;
  for (int p = 0; p < world; ++p) {
    char* base = reinterpret_cast<char*>(bases[p]);
    rs.dst[p] = base + rs_off + rank * slot_bytes;
    rs.flag[p] = reinterpret_cast<uint32_t*>(base + flag_off) + nvb::COMM_RS_FLAGS + rank;
  }
  char* mine = reinterpret_cast<char*>(bases[rank]);
  rs.calls = reinterpret_cast<const uint32_t*>(mine + flag_off) + nvb::COMM_CTRL;
  rs.ctas_done = reinterpret_cast<uint32_t*>(mine + flag_off) + nvb::COMM_CTRL_GEMM_DONE;
  at::cuda::CUDAGuard g(x.device());
  nvb::GemmPlan pl{};
  cudaError_t e = nvb::gemm_bf16_rs(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), n, m, n, k, rs,
                                    tune_out.data_ptr(), tune_out.stride(0),
                                    at::cuda::getCurrentCUDAStream().stream(), &pl);
  TORCH_CHECK(e == cudaSuccess, "gemm_bf16_rs failed: ", cudaGetErrorString(e));
  return {pl.mt, pl.bn, pl.splits};
}

// Skinny kernel (weights on the MMA's M side) with the rank-th configuration by its traffic
// model; returns (tokens per tile, weight rows per CTA, splits, stages), empty if none.
std::vector<int64_t> linear_skinny(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, int64_t rank,
                                   int64_t act, int64_t blocked, const c10::optional<at::Tensor>& trace) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16, "bf16 required");
  TORCH_CHECK(x.stride(1) == 1 && (blocked || w.stride(1) == 1) && out.stride(1) == 1, "unit inner stride required");
  const int m = (int)x.size(0), k = (int)x.size(1);
  // blocked: w is [n / 128, k / 64, 128, 64]; otherwise [n, k]
  const int n = blocked ? (int)(w.size(0) * 128) : (int)w.size(0);
  TORCH_CHECK(blocked ? (w.dim() == 4 && w.size(1) * 64 == k && w.size(2) == 128 && w.size(3) == 64 && w.is_contiguous())
                      : w.size(1) == k, "weight shape");
  TORCH_CHECK(out.size(0) == m && out.size(1) == (act ? n / 2 : n), "shape mismatch");
  nvb::GemmPlan pl{};
  if (!nvb::gemm_skinny_plan(m, n, k, (int)rank, (int)act, &pl)) return {};
  at::cuda::CUDAGuard g(x.device());
  cudaError_t e = nvb::gemm_skinny_run(x.data_ptr(), x.stride(0), w.data_ptr(), blocked ? 64 : w.stride(0),
                                       out.data_ptr(), out.stride(0), m, n, k, pl, (int)act, (int)blocked,
                                       at::cuda::getCurrentCUDAStream().stream(),
                                       trace.has_value() ? reinterpret_cast<uint64_t*>(trace->data_ptr()) : nullptr);
  TORCH_CHECK(e == cudaSuccess, "gemm_bf16 (skinny) failed: ", cudaGetErrorString(e));
  return {pl.mt, pl.bn, pl.splits, pl.stages};
}

// CTA-pair kernel (M = 256 tokens over two CTAs) with the rank-th configuration; returns
// (weight rows per pair, stages, pairs), empty if none.
std::vector<int64_t> linear_pair(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, int64_t rank, int64_t act) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16, "bf16 required");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "unit inner stride required");
  const int m = (int)x.size(0), k = (int)x.size(1), n = (int)w.size(0);
  TORCH_CHECK(w.size(1) == k && out.size(0) == m && out.size(1) == (act ? n / 2 : n), "shape mismatch");
  nvb::GemmPlan pl{};
  if (!nvb::gemm_pair_plan(m, n, k, (int)rank, (int)act, &pl)) return {};
  at::cuda::CUDAGuard g(x.device());
  cudaError_t e = nvb::gemm_bf16(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(), out.stride(0),
                                 m, n, k, pl, nullptr, nullptr, at::cuda::getCurrentCUDAStream().stream(), (int)act);
  TORCH_CHECK(e == cudaSuccess, "gemm_bf16 (pair) failed: ", cudaGetErrorString(e));
  return {pl.bn, pl.stages, pl.tiles};
}

int64_t error_code(bool reset) { return nvb::gemm_error_code(reset ? 1 : 0); }

}  // namespace

void register_gemm(pybind11::module& m) {
  m.def("linear", &linear, "tcgen05 GEMM out = x @ w^T", pybind11::arg("x"), pybind11::arg("w"),
        pybind11::arg("out"), pybind11::arg("ws") = c10::nullopt, pybind11::arg("counters") = c10::nullopt,
        pybind11::arg("force_swap") = -1,
        pybind11::arg("force_bn") = 0, pybind11::arg("force_splits") = 0, pybind11::arg("act") = 0);
  m.def("gemm_plan", &plan, pybind11::arg("m"), pybind11::arg("n"), pybind11::arg("k"),
        pybind11::arg("force_swap") = -1, pybind11::arg("force_bn") = 0, pybind11::arg("force_splits") = 0);
  m.def("linear_tuned", &linear_tuned, "autotuned tcgen05 GEMM out = x @ w^T", pybind11::arg("x"),
        pybind11::arg("w"), pybind11::arg("out"), pybind11::arg("ws") = c10::nullopt,
        pybind11::arg("counters") = c10::nullopt, pybind11::arg("act") = 0);
  m.def("linear_dec", &linear_dec, "decode-sized tcgen05 GEMM with a ranked configuration", pybind11::arg("x"),
        pybind11::arg("w"), pybind11::arg("out"), pybind11::arg("rank"), pybind11::arg("act") = 0);
  m.def("linear_dec_cfg", &linear_dec_cfg, "decode-sized tcgen05 GEMM with an explicit configuration");
  m.def("linear_skinny", &linear_skinny, "skinny tcgen05 GEMM (weights on M) with a ranked configuration",
        pybind11::arg("x"), pybind11::arg("w"), pybind11::arg("out"), pybind11::arg("rank"), pybind11::arg("act") = 0,
        pybind11::arg("blocked") = 0, pybind11::arg("trace") = c10::nullopt);
  m.def("linear_pair", &linear_pair, "CTA-pair tcgen05 GEMM (M = 256 tokens over two CTAs), ranked configuration",
        pybind11::arg("x"), pybind11::arg("w"), pybind11::arg("out"), pybind11::arg("rank"), pybind11::arg("act") = 0);
  m.def("linear_rs", &linear_rs, "tcgen05 decode GEMM whose rows are stored at their owner rank (reduce-scatter)");
  m.def("linear_sample", &linear_sample, "lm_head tcgen05 GEMM with the sampler in its epilogue", pybind11::arg("x"),
        pybind11::arg("w"), pybind11::arg("keys"), pybind11::arg("temps"), pybind11::arg("seed_step"),
        pybind11::arg("col_offset"), pybind11::arg("out_tok"), pybind11::arg("out_val") = pybind11::none(),
        pybind11::arg("ws") = pybind11::none(), pybind11::arg("counters") = pybind11::none(),
        pybind11::arg("tune") = true, pybind11::arg("force_swap") = -1, pybind11::arg("force_bn") = 0,
        pybind11::arg("force_splits") = 0);
  m.def("gemm_error", &error_code, pybind11::arg("reset") = false);
  m.def("gemm_set_deterministic", [](bool on) { nvb::gemm_set_deterministic(on ? 1 : 0); });
  m.def("gemm_deterministic", []() { return nvb::gemm_deterministic() != 0; });
}
