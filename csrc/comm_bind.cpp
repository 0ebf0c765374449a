// Python bindings of the symmetric-memory runtime and the fused TP all-reduce.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

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
                           int64_t flag_off, const at::Tensor& epochs, const at::Tensor& weight, int64_t rank,
                           int64_t rows, int64_t hidden, bool has_residual, double eps, int64_t ctas) {
  TORCH_CHECK((int)bases.size() <= nvb::COMM_MAX_RANKS, "too many ranks");
  TORCH_CHECK(weight.scalar_type() == at::kBFloat16 && weight.is_contiguous(), "weight bf16");
  TORCH_CHECK(epochs.scalar_type() == at::kInt && epochs.numel() >= ctas, "epochs int32[ctas]");
  nvb::CommArgs a;
  std::memset(&a, 0, sizeof(a));
  for (size_t p = 0; p < bases.size(); ++p) {
    char* base = reinterpret_cast<char*>(bases[p]);
    a.in[p] = reinterpret_cast<__nv_bfloat16*>(base + in_off);
    a.res[p] = reinterpret_cast<__nv_bfloat16*>(base + res_off);
    a.out[p] = reinterpret_cast<__nv_bfloat16*>(base + out_off);
    a.flags[p] = reinterpret_cast<uint32_t*>(base + flag_off);
  }
  a.epochs = reinterpret_cast<uint32_t*>(epochs.data_ptr<int>());
  a.weight = reinterpret_cast<const __nv_bfloat16*>(weight.data_ptr());
  a.rank = (int)rank;
  a.world = (int)bases.size();
  a.rows = (int)rows;
  a.hidden = (int)hidden;
  a.ctas = (int)ctas;
  a.has_residual = has_residual ? 1 : 0;
  a.eps = (float)eps;
  at::cuda::CUDAGuard g(weight.device());
  check(nvb::launch_allreduce_add_rmsnorm(a, at::cuda::getCurrentCUDAStream().stream()), "allreduce_add_rmsnorm");
}

int64_t comm_error(bool reset) { return nvb::comm_error_code(reset ? 1 : 0); }

}  // namespace

void register_comm(pybind11::module& m) {
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_free", &symm_free);
  m.def("allreduce_add_rmsnorm", &allreduce_add_rmsnorm);
  m.def("comm_error", &comm_error, pybind11::arg("reset") = false);
  m.attr("COMM_FLAG_BYTES") = (int64_t)nvb::COMM_FLAG_BYTES;
  m.attr("COMM_MAX_CTAS") = (int64_t)nvb::COMM_MAX_CTAS;
}
