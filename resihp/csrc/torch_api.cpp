// Torch-facing wrappers and Python bindings of the sm_100a kernels (module resihp._C).
// Shapes, dtypes and strides are checked here; the CUDA launchers behind launch.h only
// see raw pointers, so the kernel translation units stay free of torch headers.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>

#include "launch.h"

namespace resihp {

// ---- error word ---------------------------------------------------------------------

static int* g_error_words[64] = {nullptr};
static std::mutex g_error_mutex;

int* error_word(const c10::Device& device) {
  const int idx = device.index() < 0 ? 0 : device.index();
  TORCH_CHECK(idx < 64, "device index out of range");
  if (g_error_words[idx] == nullptr) {
    std::lock_guard<std::mutex> lock(g_error_mutex);
    if (g_error_words[idx] == nullptr) {
      c10::cuda::CUDAGuard guard(device);
      int* p = nullptr;
      C10_CUDA_CHECK(cudaMalloc(&p, sizeof(int)));
      C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
      g_error_words[idx] = p;
    }
  }
  return g_error_words[idx];
}

// Synchronising read of the device's error word; resets it to zero.
int64_t read_and_clear_error(int64_t device_index) {
  const c10::Device dev(c10::kCUDA, device_index);
  int* p = error_word(dev);
  c10::cuda::CUDAGuard guard(dev);
  auto stream = at::cuda::getCurrentCUDAStream();
  int value = 0;
  C10_CUDA_CHECK(cudaMemcpyAsync(&value, p, sizeof(int), cudaMemcpyDeviceToHost, stream));
  C10_CUDA_CHECK(cudaStreamSynchronize(stream));
  if (value != 0) C10_CUDA_CHECK(cudaMemsetAsync(p, 0, sizeof(int), stream));
  return value;
}

static cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

static void check_cuda_bf16(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bf16");
}

// ---- GEMM ---------------------------------------------------------------------------

void gemm(torch::Tensor a, bool a_mn, torch::Tensor b, bool b_mn, torch::Tensor c, int64_t epi, double alpha,
          c10::optional<torch::Tensor> residual, int64_t max_ctas, int64_t force_bn) {
  check_cuda_bf16(a, "A");
  check_cuda_bf16(b, "B");
  TORCH_CHECK(c.is_cuda(), "C must be a CUDA tensor");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "GEMM operands must be 2-D");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && c.stride(1) == 1, "GEMM operands need unit inner stride");
  const int64_t m = a_mn ? a.size(1) : a.size(0);
  const int64_t k = a_mn ? a.size(0) : a.size(1);
  const int64_t n = b_mn ? b.size(1) : b.size(0);
  const int64_t kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(k == kb, "GEMM reduction sizes differ: ", k, " vs ", kb);
  TORCH_CHECK(c.size(0) == m && c.size(1) == n, "GEMM output shape mismatch");
  const bool want_f32 = epi == 1 || epi == 2;
  TORCH_CHECK(c.scalar_type() == (want_f32 ? at::kFloat : at::kBFloat16), "GEMM output dtype does not match epilogue");
  const void* r = nullptr;
  int64_t ldr = 0;
  if (epi == 3) {
    TORCH_CHECK(residual.has_value(), "residual epilogue needs a residual tensor");
    const auto& rt = *residual;
    check_cuda_bf16(rt, "residual");
    TORCH_CHECK(rt.size(0) == m && rt.size(1) == n && rt.stride(1) == 1, "residual must be [m, n]");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(rt.data_ptr()) % 16 == 0 && rt.stride(0) % 8 == 0, "residual alignment");
    r = rt.data_ptr();
    ldr = rt.stride(0);
  }
  TORCH_CHECK(m <= INT32_MAX && n <= INT32_MAX && k <= INT32_MAX, "GEMM too large");
  c10::cuda::CUDAGuard guard(a.device());
  gemm_raw(a.data_ptr(), a.stride(0), a_mn, b.data_ptr(), b.stride(0), b_mn, c.data_ptr(), c.stride(0), r, ldr,
           int(m), int(n), int(k), int(epi), float(alpha), error_word(a.device()), cur_stream(), int(max_ctas),
           int(force_bn));
}

}  // namespace resihp

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "resihp sm_100a kernels";
  m.def("read_and_clear_error", &resihp::read_and_clear_error, "synchronising read+reset of the kernel error word");
  m.def("gemm", &resihp::gemm, "tcgen05 bf16 GEMM", py::arg("a"), py::arg("a_mn"), py::arg("b"), py::arg("b_mn"),
        py::arg("c"), py::arg("epi"), py::arg("alpha") = 1.0, py::arg("residual") = py::none(),
        py::arg("max_ctas") = 0, py::arg("force_bn") = 0);
}
