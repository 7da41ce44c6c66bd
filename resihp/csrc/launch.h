// Torch-free host interface of the CUDA kernels. Each launcher validates its arguments,
// enqueues on ``stream`` and throws std::runtime_error on misuse; the torch-facing
// wrappers in torch_api.cpp translate tensors into these calls.
#pragma once
#include <cstdint>
#include <sstream>
#include <stdexcept>
#include <cuda.h>
#include <cuda_runtime.h>

namespace resihp {

namespace detail {
inline void append(std::ostringstream&) {}
template <class T, class... R>
inline void append(std::ostringstream& o, const T& v, const R&... r) {
  o << v;
  append(o, r...);
}
}  // namespace detail

#define RESIHP_CHECK(cond, ...)                                                        \
  do {                                                                                 \
    if (!(cond)) {                                                                     \
      std::ostringstream _o;                                                           \
      ::resihp::detail::append(_o, "resihp: ", __VA_ARGS__);                           \
      throw std::runtime_error(_o.str());                                              \
    }                                                                                  \
  } while (0)

#define RESIHP_CUDA_CHECK(expr)                                                        \
  do {                                                                                 \
    cudaError_t _e = (expr);                                                           \
    RESIHP_CHECK(_e == cudaSuccess, #expr, " failed: ", cudaGetErrorString(_e));        \
  } while (0)

CUtensorMap make_tma_2d_bf16(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_cols, int box_rows);

// C[m,n] (=, +=) alpha * A * B^T; see gemm.cu for operand conventions and epilogues.
void gemm_raw(const void* a, int64_t lda, bool a_mn, const void* b, int64_t ldb, bool b_mn, void* c, int64_t ldc,
              const void* r, int64_t ldr, int m, int n, int k, int epi, float alpha, int* err, cudaStream_t stream,
              int max_ctas, int force_bn);

}  // namespace resihp
