// Python bindings of the symmetric-memory runtime and the fused TP all-reduce.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>
#include <cstring>

#include "comm.h"

namespace {

void check(cudaError_t e, const char* what) { TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e)); }

// Allocate `bytes` of IPC-shareable device memory; returns (pointer, 64-byte handle).
std::tuple<int64_t, py::bytes> symm_alloc(int64_t bytes) {
  void* p = nullptr;
  char h[64];
  check(nvb::symm_alloc((size_t)bytes, &p, h), "symm_alloc");
  return {reinterpret_cast<int64_t>(p), py::bytes(h, 64)};
}

int64_t symm_open(py::bytes handle) {
  std::string s = handle;
  TORCH_CHECK(s.size() == 64, "IPC handle must be 64 bytes");
  void* p = nullptr;
  check(nvb::symm_open(s.data(), &p), "symm_open");
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t p) { check(nvb::symm_close(reinterpret_cast<void*>(p)), "symm_close"); }
void symm_free(int64_t p) { check(nvb::symm_free(reinterpret_cast<void*>(p)), "symm_free"); }

// bases[p] = rank p's buffer (opened locally); layout offsets in bytes.
void allreduce_add_rmsnorm(std::vector<int64_t> bases, int64_t in_off, int64_t res_off, int64_t out_off,
                           int64_t flag_off, const at::Tensor& weight, int64_t rank,
                           int64_t rows, int64_t hidden, bool has_residual, double eps, int64_t ctas,
                           bool oneshot, int64_t timeout_ns) {
  TORCH_CHECK((int)bases.size() <= nvb::COMM_MAX_RANKS, "too many ranks");
  TORCH_CHECK(weight.scalar_type() == at::kBFloat16 && weight.is_contiguous(), "weight bf16");
  nvb::CommArgs a;
  std::memset(&a, 0, sizeof(a));
  for (size_t p = 0; p < bases.size(); ++p) {
    char* base = reinterpret_cast<char*>(bases[p]);
    a.in[p] = reinterpret_cast<__nv_bfloat16*>(base + in_off);
    a.res[p] = reinterpret_cast<__nv_bfloat16*>(base + res_off);
    a.out[p] = reinterpret_cast<__nv_bfloat16*>(base + out_off);
    a.flags[p] = reinterpret_cast<uint32_t*>(base + flag_off);
  }
  a.weight = reinterpret_cast<const __nv_bfloat16*>(weight.data_ptr());
  a.rank = (int)rank;
  a.world = (int)bases.size();
  a.rows = (int)rows;
  a.hidden = (int)hidden;
  a.ctas = (int)ctas;
  a.has_residual = has_residual ? 1 : 0;
  a.timeout_ns = (uint64_t)(timeout_ns > 0 ? timeout_ns : 0);
  a.eps = (float)eps;
  at::cuda::CUDAGuard g(weight.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
  check(oneshot ? nvb::launch_allreduce_oneshot(a, st) : nvb::launch_allreduce_add_rmsnorm(a, st),
        "allreduce_add_rmsnorm");
}

// Owner side of the GEMM -> reduce-scatter path (RsNormArgs): rs_off = this rank's receive
// area, res_off / out_off / flag_off as in allreduce_add_rmsnorm.
void rs_add_rmsnorm_ag(std::vector<int64_t> bases, int64_t rs_off, int64_t res_off, int64_t out_off, int64_t flag_off,
                       const at::Tensor& weight, int64_t rank, int64_t rows, int64_t rs_rows, int64_t hidden,
                       bool has_residual, double eps, int64_t ctas, int64_t timeout_ns) {
  TORCH_CHECK((int)bases.size() <= nvb::COMM_MAX_RANKS, "too many ranks");
  TORCH_CHECK(rank >= 0 && rank < (int64_t)bases.size(), "rank out of range");
  TORCH_CHECK(weight.scalar_type() == at::kBFloat16 && weight.is_contiguous(), "weight bf16");
  nvb::RsNormArgs a;
  std::memset(&a, 0, sizeof(a));
  for (size_t p = 0; p < bases.size(); ++p) {
    char* base = reinterpret_cast<char*>(bases[p]);
    a.out[p] = reinterpret_cast<__nv_bfloat16*>(base + out_off);
    a.flags[p] = reinterpret_cast<uint32_t*>(base + flag_off);
  }
  char* mine = reinterpret_cast<char*>(bases[rank]);
  a.rs = reinterpret_cast<const __nv_bfloat16*>(mine + rs_off);
  a.res = reinterpret_cast<__nv_bfloat16*>(mine + res_off);
  a.weight = reinterpret_cast<const __nv_bfloat16*>(weight.data_ptr());
  a.rank = (int)rank;
  a.world = (int)bases.size();
  a.rows = (int)rows;
  a.rs_rows = (int)rs_rows;
  a.hidden = (int)hidden;
  a.ctas = (int)ctas;
  a.has_residual = has_residual ? 1 : 0;
  a.timeout_ns = (uint64_t)(timeout_ns > 0 ? timeout_ns : 0);
  a.eps = (float)eps;
  at::cuda::CUDAGuard g(weight.device());
  check(nvb::launch_rs_add_rmsnorm_ag(a, at::cuda::getCurrentCUDAStream().stream()), "rs_add_rmsnorm_ag");
}

int64_t comm_error(bool reset) { return nvb::comm_error_code(reset ? 1 : 0); }

// Push blocks of a local KV pool [2, L, NB, ...] into a peer pool (raw pointer, nb_dst blocks).
void kv_push(const at::Tensor& pool, const at::Tensor& src_ids, const at::Tensor& dst_ids, int64_t dst_ptr,
             int64_t nb_dst) {
  TORCH_CHECK(pool.is_cuda() && pool.is_contiguous() && pool.dim() >= 3, "pool [2, L, NB, ...] contiguous");
  TORCH_CHECK(src_ids.scalar_type() == at::kInt && dst_ids.scalar_type() == at::kInt, "int32 ids");
  TORCH_CHECK(src_ids.numel() == dst_ids.numel(), "id count mismatch");
  const int planes = (int)(pool.size(0) * pool.size(1));
  const int nb_src = (int)pool.size(2);
  const int64_t block_bytes = pool.numel() / ((int64_t)planes * nb_src) * pool.element_size();
  at::cuda::CUDAGuard g(pool.device());
  check(nvb::launch_kv_push(pool.data_ptr(), reinterpret_cast<void*>(dst_ptr), src_ids.data_ptr<int>(),
                            dst_ids.data_ptr<int>(), (int)src_ids.numel(), planes, nb_src, (int)nb_dst, block_bytes,
                            at::cuda::getCurrentCUDAStream().stream()),
        "kv_push");
}

// Raise a peer's push flag (raw pointer into its exported allocation) to `epoch`, in stream
// order after the pushes launched before.
void kv_push_signal(int64_t flag_ptr, int64_t epoch) {
  check(nvb::launch_push_signal(reinterpret_cast<uint32_t*>(flag_ptr), (uint32_t)epoch,
                                at::cuda::getCurrentCUDAStream().stream()),
        "kv_push_signal");
}

// Make the current stream wait until this device's push flag word reaches `epoch`; `status`
// (int32, optional) receives 1 on arrival, 2 when the bounded wait gave up.
void kv_push_wait(int64_t flag_ptr, int64_t epoch, int64_t timeout_ns, const c10::optional<at::Tensor>& status) {
  int* st = nullptr;
  if (status.has_value()) {
    TORCH_CHECK(status->is_cuda() && status->scalar_type() == at::kInt && status->numel() >= 1, "status int32");
    st = status->data_ptr<int>();
  }
  check(nvb::launch_push_wait(reinterpret_cast<const uint32_t*>(flag_ptr), (uint32_t)epoch, (uint64_t)timeout_ns, st,
                              at::cuda::getCurrentCUDAStream().stream()),
        "kv_push_wait");
}

int64_t push_error(bool reset) { return nvb::push_error_code(reset ? 1 : 0); }

}  // namespace

void register_comm(pybind11::module& m) {
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_free", &symm_free);
  m.def("allreduce_add_rmsnorm", &allreduce_add_rmsnorm, pybind11::arg("bases"), pybind11::arg("in_off"),
        pybind11::arg("res_off"), pybind11::arg("out_off"), pybind11::arg("flag_off"),
        pybind11::arg("weight"), pybind11::arg("rank"), pybind11::arg("rows"), pybind11::arg("hidden"),
        pybind11::arg("has_residual"), pybind11::arg("eps"), pybind11::arg("ctas"), pybind11::arg("oneshot") = false,
        pybind11::arg("timeout_ns") = 0);
  m.def("rs_add_rmsnorm_ag", &rs_add_rmsnorm_ag, pybind11::arg("bases"), pybind11::arg("rs_off"),
        pybind11::arg("res_off"), pybind11::arg("out_off"), pybind11::arg("flag_off"), pybind11::arg("weight"),
        pybind11::arg("rank"), pybind11::arg("rows"), pybind11::arg("rs_rows"), pybind11::arg("hidden"),
        pybind11::arg("has_residual"), pybind11::arg("eps"), pybind11::arg("ctas"), pybind11::arg("timeout_ns") = 0);
  m.def("comm_error", &comm_error, pybind11::arg("reset") = false);
  m.def("kv_push", &kv_push);
  m.def("kv_push_signal", &kv_push_signal);
  m.def("kv_push_wait", &kv_push_wait, pybind11::arg("flag_ptr"), pybind11::arg("epoch"),
        pybind11::arg("timeout_ns") = 0, pybind11::arg("status") = pybind11::none());
  m.def("push_error", &push_error, pybind11::arg("reset") = false);
  m.attr("PUSH_FLAG_SLOTS") = (int64_t)nvb::PUSH_FLAG_SLOTS;
  m.attr("COMM_FLAG_BYTES") = (int64_t)nvb::COMM_FLAG_BYTES;
  m.attr("COMM_MAX_CTAS") = (int64_t)nvb::COMM_MAX_CTAS;
  m.attr("COMM_RS_MAX_ROWS") = (int64_t)nvb::COMM_RS_MAX_ROWS;
}
