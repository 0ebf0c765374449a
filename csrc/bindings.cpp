// Python bindings (torch tensors -> raw launches on the current CUDA stream).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "kernels.h"

namespace {

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bfloat16")
#define CHECK_I32(x) TORCH_CHECK((x).scalar_type() == at::kInt, #x " must be int32")

void check(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, " failed: ", cudaGetErrorString(e));
}

template <typename T>
T* ptr_or_null(const c10::optional<at::Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void add_rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual_in,
                 const c10::optional<at::Tensor>& residual_out, const at::Tensor& w, at::Tensor& out, double eps,
                 const c10::optional<at::Tensor>& row_index) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  CHECK_BF16(out);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be [rows, H] with unit inner stride");
  int H = (int)x.size(1);
  int rows = (int)out.size(0);
  if (row_index.has_value()) CHECK_I32(*row_index);
  if (residual_in.has_value()) CHECK_CONTIG(*residual_in);
  at::cuda::CUDAGuard g(x.device());
  check(nvb::launch_add_rmsnorm(x.data_ptr(), x.stride(0), ptr_or_null<void>(residual_in),
                                ptr_or_null<void>(residual_out), w.data_ptr(), out.data_ptr(), rows, H, (float)eps,
                                ptr_or_null<int>(row_index), stream(), (int)x.size(0)),
        "add_rmsnorm");
}

void silu_mul(const at::Tensor& x, at::Tensor& out) {
  CHECK_CONTIG(x);
  CHECK_BF16(x);
  CHECK_CONTIG(out);
  at::cuda::CUDAGuard g(x.device());
  check(nvb::launch_silu_mul(x.data_ptr(), out.data_ptr(), (int)x.size(0), (int)out.size(1), stream()), "silu_mul");
}

void embedding(const at::Tensor& ids, const at::Tensor& table, int64_t vocab_start, at::Tensor& out) {
  CHECK_I32(ids);
  CHECK_CONTIG(table);
  CHECK_BF16(table);
  at::cuda::CUDAGuard g(ids.device());
  check(nvb::launch_embedding(ids.data_ptr<int>(), table.data_ptr(), (int)table.size(0), (int)vocab_start,
                              out.data_ptr(), (int)ids.size(0), (int)table.size(1), stream()),
        "embedding");
}

void qkv_post(const at::Tensor& qkv, at::Tensor& q_out, const at::Tensor& q_norm, const at::Tensor& k_norm, double eps,
              const at::Tensor& positions, const at::Tensor& cos_sin, at::Tensor& k_cache, at::Tensor& v_cache,
              const c10::optional<at::Tensor>& k_scale, const c10::optional<at::Tensor>& v_scale,
              const at::Tensor& slots, int64_t nq, int64_t nkv) {
  CHECK_BF16(qkv);
  TORCH_CHECK(qkv.stride(1) == 1, "qkv inner stride");
  CHECK_I32(positions);
  CHECK_I32(slots);
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous(), "cos_sin fp32 contiguous");
  int fp8 = k_cache.scalar_type() == at::kFloat8_e4m3fn;
  TORCH_CHECK(fp8 || k_cache.scalar_type() == at::kBFloat16, "KV cache must be bf16 or fp8 e4m3");
  TORCH_CHECK(!fp8 || (k_scale.has_value() && v_scale.has_value()), "fp8 KV cache needs scales");
  at::cuda::CUDAGuard g(qkv.device());
  check(nvb::launch_qkv_post(qkv.data_ptr(), qkv.stride(0), q_out.data_ptr(), q_norm.data_ptr(), k_norm.data_ptr(),
                             (float)eps, positions.data_ptr<int>(), cos_sin.data_ptr<float>(), k_cache.data_ptr(),
                             v_cache.data_ptr(), ptr_or_null<float>(k_scale), ptr_or_null<float>(v_scale),
                             slots.data_ptr<int>(), (int)qkv.size(0), (int)nq, (int)nkv, (int)k_cache.size(3),
                             (int)k_cache.size(2), fp8, stream(), (int)k_cache.size(0)),
        "qkv_post");
}

nvb::AttnLaunch attn_args(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                          const c10::optional<at::Tensor>& k_scale, const c10::optional<at::Tensor>& v_scale,
                          const at::Tensor& block_tables, const at::Tensor& cu_q, const at::Tensor& ctx_lens,
                          at::Tensor& out, int64_t nq, int64_t nkv, int64_t seq_offset, int64_t num_seqs,
                          double scale) {
  CHECK_BF16(q);
  CHECK_CONTIG(q);
  CHECK_CONTIG(k_cache);
  CHECK_CONTIG(v_cache);
  CHECK_I32(block_tables);
  CHECK_CONTIG(block_tables);
  CHECK_I32(cu_q);
  CHECK_I32(ctx_lens);
  int fp8 = k_cache.scalar_type() == at::kFloat8_e4m3fn;
  TORCH_CHECK(fp8 || k_cache.scalar_type() == at::kBFloat16, "KV cache must be bf16 or fp8 e4m3");
  nvb::AttnLaunch L{};
  L.q = q.data_ptr();
  L.k_cache = k_cache.data_ptr();
  L.v_cache = v_cache.data_ptr();
  L.k_scale = ptr_or_null<float>(k_scale);
  L.v_scale = ptr_or_null<float>(v_scale);
  L.block_tables = block_tables.data_ptr<int>();
  L.W = (int)block_tables.size(1);
  L.cu_q = cu_q.data_ptr<int>();
  L.ctx_lens = ctx_lens.data_ptr<int>();
  L.out = out.data_ptr();
  L.nq = (int)nq;
  L.nkv = (int)nkv;
  L.head_dim = (int)k_cache.size(3);
  L.block_size = (int)k_cache.size(2);
  L.num_blocks = (int)k_cache.size(0);
  L.seq_offset = (int)seq_offset;
  L.num_seqs = (int)num_seqs;
  L.kv_fp8 = fp8;
  L.softmax_scale = (float)scale;
  return L;
}

void attn_decode(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                 const c10::optional<at::Tensor>& k_scale, const c10::optional<at::Tensor>& v_scale,
                 const at::Tensor& block_tables, const at::Tensor& cu_q, const at::Tensor& ctx_lens, at::Tensor& out,
                 const c10::optional<at::Tensor>& part_o, const c10::optional<at::Tensor>& part_lse, int64_t nq,
                 int64_t nkv, int64_t splits, int64_t seq_offset, int64_t num_seqs, double scale) {
  auto L = attn_args(q, k_cache, v_cache, k_scale, v_scale, block_tables, cu_q, ctx_lens, out, nq, nkv, seq_offset,
                     num_seqs, scale);
  L.splits = (int)splits;
  L.part_o = ptr_or_null<float>(part_o);
  L.part_lse = ptr_or_null<float>(part_lse);
  if (splits > 1) {
    TORCH_CHECK(part_o.has_value() && part_lse.has_value(), "split decode needs scratch");
    int64_t need = (seq_offset + num_seqs) * nq * splits;
    TORCH_CHECK(part_lse->numel() >= need && part_o->numel() >= need * L.head_dim, "decode scratch too small");
  }
  at::cuda::CUDAGuard g(q.device());
  check(nvb::launch_attn_decode(L, stream()), "attn_decode");
}

void attn_prefill(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                  const c10::optional<at::Tensor>& k_scale, const c10::optional<at::Tensor>& v_scale,
                  const at::Tensor& block_tables, const at::Tensor& cu_q, const at::Tensor& ctx_lens, at::Tensor& out,
                  int64_t nq, int64_t nkv, int64_t seq_offset, int64_t num_seqs, int64_t max_q_len, double scale,
                  int64_t use_tc) {
  auto L = attn_args(q, k_cache, v_cache, k_scale, v_scale, block_tables, cu_q, ctx_lens, out, nq, nkv, seq_offset,
                     num_seqs, scale);
  L.splits = 1;
  at::cuda::CUDAGuard g(q.device());
  check(nvb::launch_attn_prefill_ex(L, (int)max_q_len, (int)q.size(0), (int)use_tc, stream()), "attn_prefill");
}

int64_t decode_splits(int64_t num_seqs, int64_t nkv, int64_t max_ctx, int64_t num_sms) {
  return nvb::attn_decode_splits((int)num_seqs, (int)nkv, (int)max_ctx, (int)num_sms);
}

int64_t attn_error(bool reset) { return nvb::attn_error_code(reset ? 1 : 0); }

int64_t sample_chunks(int64_t rows, int64_t V) { return nvb::sample_num_chunks((int)rows, (int)V); }

void sample(const at::Tensor& logits, int64_t col_offset, const at::Tensor& temps, const at::Tensor& seed_step,
            at::Tensor& part_val, at::Tensor& part_idx, int64_t nchunk, at::Tensor& out_tok,
            const c10::optional<at::Tensor>& out_val) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits [rows, V]");
  TORCH_CHECK(temps.scalar_type() == at::kFloat, "temps fp32");
  TORCH_CHECK(seed_step.scalar_type() == at::kLong && seed_step.numel() >= 2, "seed_step int64[2]");
  TORCH_CHECK(part_val.numel() >= logits.size(0) * nchunk && part_idx.numel() >= logits.size(0) * nchunk,
              "sample scratch too small");
  int bf16 = logits.scalar_type() == at::kBFloat16;
  TORCH_CHECK(bf16 || logits.scalar_type() == at::kFloat, "logits bf16 or fp32");
  at::cuda::CUDAGuard g(logits.device());
  check(nvb::launch_sample(logits.data_ptr(), bf16, logits.stride(0), (int)logits.size(0), (int)logits.size(1),
                           col_offset, temps.data_ptr<float>(), seed_step.data_ptr<int64_t>(),
                           part_val.data_ptr<float>(), part_idx.data_ptr<int>(), (int)nchunk, out_tok.data_ptr<int>(),
                           ptr_or_null<float>(out_val), stream()),
        "sample");
}

// Row-parallel sampler (greedy / temperature / top-p); with xbases / fbases (every rank's
// exchange and flag areas of the symmetric buffer, as integers) the vocabulary shards of a
// tensor-parallel group are combined inside the kernel.
void sample_rows(const at::Tensor& logits, int64_t col_offset, const at::Tensor& temps,
                 const c10::optional<at::Tensor>& top_p, const at::Tensor& seed_step, at::Tensor& out_tok,
                 const c10::optional<at::Tensor>& out_val, std::vector<int64_t> xbases, std::vector<int64_t> fbases,
                 int64_t rank, int64_t rows_cap, int64_t timeout_ns) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits [rows, V]");
  TORCH_CHECK(temps.scalar_type() == at::kFloat, "temps fp32");
  TORCH_CHECK(!top_p.has_value() || top_p->scalar_type() == at::kFloat, "top_p fp32");
  TORCH_CHECK(seed_step.scalar_type() == at::kLong && seed_step.numel() >= 2, "seed_step int64[2]");
  TORCH_CHECK(xbases.size() == fbases.size() && xbases.size() <= 8, "exchange areas");
  int bf16 = logits.scalar_type() == at::kBFloat16;
  TORCH_CHECK(bf16 || logits.scalar_type() == at::kFloat, "logits bf16 or fp32");
  nvb::SampleX X;
  if (xbases.size() > 1) {
    X.world = (int)xbases.size();
    X.rank = (int)rank;
    X.rows_cap = (int)rows_cap;
    for (size_t p = 0; p < xbases.size(); ++p) {
      X.x[p] = reinterpret_cast<float*>(xbases[p]);
      X.f[p] = reinterpret_cast<uint32_t*>(fbases[p]);
    }
    X.ctrl = X.f[rank] + 4LL * rows_cap * X.world;
    if (timeout_ns > 0) X.timeout_ns = (uint64_t)timeout_ns;
  }
  at::cuda::CUDAGuard g(logits.device());
  check(nvb::launch_sample_rows(logits.data_ptr(), bf16, logits.stride(0), (int)logits.size(0), (int)logits.size(1),
                                col_offset, temps.data_ptr<float>(), ptr_or_null<float>(top_p),
                                seed_step.data_ptr<int64_t>(), out_tok.data_ptr<int>(), ptr_or_null<float>(out_val), X,
                                stream()),
        "sample_rows");
}

int64_t sample_x_floats(int64_t world, int64_t rows_cap) { return nvb::sample_x_floats((int)world, (int)rows_cap); }
int64_t sample_f_words(int64_t world, int64_t rows_cap) { return nvb::sample_f_words((int)world, (int)rows_cap); }
int64_t sample_error(bool reset) { return nvb::sample_error_code(reset ? 1 : 0); }

// First index-check error recorded by the checked kernels (401: gathered norm row out of range,
// 402: KV slot beyond the pool, 403: a q/k/v stage copy did not arrive in time), 0 if none.
int64_t bounds_error(bool reset) {
  const int a = nvb::norm_check_code(reset ? 1 : 0);
  const int b = nvb::qkv_check_code(reset ? 1 : 0);
  return a ? a : b;
}

}  // namespace

void register_gemm(pybind11::module& m);
void register_comm(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "nanovllm_self_b200 sm_100a kernels";
  m.def("add_rmsnorm", &add_rmsnorm);
  m.def("silu_mul", &silu_mul);
  m.def("embedding", &embedding);
  m.def("qkv_post", &qkv_post);
  m.def("attn_decode", &attn_decode);
  m.def("attn_prefill", &attn_prefill, pybind11::arg("q"), pybind11::arg("k_cache"), pybind11::arg("v_cache"),
        pybind11::arg("k_scale"), pybind11::arg("v_scale"), pybind11::arg("block_tables"), pybind11::arg("cu_q"),
        pybind11::arg("ctx_lens"), pybind11::arg("out"), pybind11::arg("nq"), pybind11::arg("nkv"),
        pybind11::arg("seq_offset"), pybind11::arg("num_seqs"), pybind11::arg("max_q_len"), pybind11::arg("scale"),
        pybind11::arg("use_tc") = 1);
  m.def("decode_splits", &decode_splits);
  m.def("attn_error", &attn_error, pybind11::arg("reset") = false);
  m.def("sample_chunks", &sample_chunks);
  m.def("sample", &sample);
  m.def("sample_rows", &sample_rows, pybind11::arg("logits"), pybind11::arg("col_offset"), pybind11::arg("temps"),
        pybind11::arg("top_p"), pybind11::arg("seed_step"), pybind11::arg("out_tok"), pybind11::arg("out_val"),
        pybind11::arg("xbases") = std::vector<int64_t>{}, pybind11::arg("fbases") = std::vector<int64_t>{},
        pybind11::arg("rank") = 0, pybind11::arg("rows_cap") = 0, pybind11::arg("timeout_ns") = 0);
  m.def("sample_x_floats", &sample_x_floats);
  m.def("sample_f_words", &sample_f_words);
  m.def("sample_rows_capacity", &nvb::sample_rows_capacity);
  m.def("sample_error", &sample_error, pybind11::arg("reset") = false);
  m.def("bounds_error", &bounds_error, pybind11::arg("reset") = false);
  m.attr("BOUNDS_CHECK") = (int64_t)nvb::bounds_check_enabled();
  register_gemm(m);
  register_comm(m);
}
