// Python bindings of the sm_100a kernels.  Kernel files (*.cu) include no torch headers;
// this file turns tensors into raw pointers, picks the current stream and reports errors.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>
#include <unordered_map>

#include "kernels.h"

namespace {

// One error word per device, written by kernels whose bounded waits ran out.
torch::Tensor& error_word(int device) {
  static std::mutex mu;
  static std::unordered_map<int, torch::Tensor> words;
  std::lock_guard<std::mutex> g(mu);
  auto it = words.find(device);
  if (it == words.end()) {
    auto t = torch::zeros({4}, torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, device));
    it = words.emplace(device, t).first;
  }
  return it->second;
}

int* err_ptr(const torch::Tensor& like) { return error_word(like.get_device()).data_ptr<int>(); }

int num_sms(int device) {
  static std::mutex mu;
  static std::unordered_map<int, int> cache;
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(device);
  if (it != cache.end()) return it->second;
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  cache[device] = n;
  return n;
}

void check_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

// Leading dimension of a 2-D operand whose inner dimension is contiguous.
long long ld_of(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must have a contiguous inner dimension");
  return t.size(0) > 1 ? t.stride(0) : t.size(1);
}

}  // namespace

// out[M,N] (+)= alpha * op(a) @ op(b)^T ; a is [M,K] (or [K,M] if a_t), b is [N,K] (or [K,N] if b_t)
void gemm(const torch::Tensor& a, bool a_t, const torch::Tensor& b, bool b_t, torch::Tensor& out,
          int64_t epi, double alpha, const c10::optional<torch::Tensor>& residual) {
  check_cuda(a, "a");
  check_cuda(b, "b");
  check_cuda(out, "out");
  TORCH_CHECK(a.scalar_type() == torch::kBFloat16 && b.scalar_type() == torch::kBFloat16,
              "gemm operands must be bf16");
  const long long lda = ld_of(a, "a"), ldb = ld_of(b, "b"), ldd = ld_of(out, "out");
  const int M = a_t ? a.size(1) : a.size(0);
  const int K = a_t ? a.size(0) : a.size(1);
  const int N = b_t ? b.size(1) : b.size(0);
  const int Kb = b_t ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm: contraction sizes differ (", K, " vs ", Kb, ")");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm: out must be [", M, ", ", N, "]");
  if (epi == 1 || epi == 2) {
    TORCH_CHECK(out.scalar_type() == torch::kFloat32, "fp32 epilogue needs an fp32 output");
  } else {
    TORCH_CHECK(out.scalar_type() == torch::kBFloat16, "bf16 epilogue needs a bf16 output");
  }
  const void* rptr = nullptr;
  long long ldr = 0;
  if (epi == 3) {
    TORCH_CHECK(residual.has_value(), "residual epilogue needs a residual");
    const auto& r = *residual;
    TORCH_CHECK(r.scalar_type() == torch::kBFloat16 && r.size(0) == M && r.size(1) == N, "bad residual");
    rptr = r.data_ptr();
    ldr = ld_of(r, "residual");
  }
  const c10::cuda::CUDAGuard guard(a.device());
  if (K == 0) {
    if (epi == 2) return;
    out.zero_();
    if (epi == 3) out.copy_(*residual);
    return;
  }
  const int rc = rb::gemm_bf16(a.data_ptr(), lda, a_t, b.data_ptr(), ldb, b_t, out.data_ptr(), ldd, rptr, ldr,
                               M, N, K, static_cast<int>(epi), static_cast<float>(alpha), err_ptr(a),
                               num_sms(a.get_device()), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "gemm_bf16 failed with code ", rc);
}

torch::Tensor error_state(int64_t device) { return error_word(static_cast<int>(device)); }

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of resihp_megatron_b200";
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM", py::arg("a"), py::arg("a_t"), py::arg("b"), py::arg("b_t"),
        py::arg("out"), py::arg("epi"), py::arg("alpha"), py::arg("residual") = py::none());
  m.def("error_state", &error_state, "per-device kernel error words");
}
