// RMSNorm forward/backward (bf16 activations, fp32 statistics), with the residual add of
// a pre-norm block fused in (the Llama counterpart of the reference's ``F.layer_norm``
// calls, resihp/parallel/tp.py:262,264,268, and their residual adds):
//
//   forward   s = x (+ r);   y = s * rstd * w,   rstd = 1 / sqrt(mean(s^2) + eps)
//   backward  g = dy * w;    ds = rstd * (g - s_hat * mean(g * s_hat)) (+ dres),
//             dw += sum_rows dy * s_hat                  (s_hat = s * rstd)
//
// One row is spread over d/8 threads, each holding one 16-byte vector (8 bf16); several
// rows share a block so that a block has >= 256 threads. The weight gradient is
// reduced deterministically: every block of a fixed-size persistent grid writes one
// fp32 partial row, and a second kernel sums the partials in block order.
#include <cuda_bf16.h>

#include "common.cuh"
#include "launch.h"

namespace resihp {

namespace {

struct Vec8 {
  float v[8];
};

__device__ __forceinline__ Vec8 load8(const __nv_bfloat16* p) {
  uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  Vec8 out;
  #pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    out.v[2 * i] = f.x;
    out.v[2 * i + 1] = f.y;
  }
  return out;
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const Vec8& x) {
  uint4 raw;
  raw.x = pack_bf16(x.v[0], x.v[1]);
  raw.y = pack_bf16(x.v[2], x.v[3]);
  raw.z = pack_bf16(x.v[4], x.v[5]);
  raw.w = pack_bf16(x.v[6], x.v[7]);
  *reinterpret_cast<uint4*>(p) = raw;
}

// Sum over the `lanes` threads (a power of two, or a multiple of 32) sharing one row.
// `scratch` holds one float per warp of the block.
__device__ __forceinline__ float row_sum(float v, int lanes, float* scratch) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    if (o < lanes) v += __shfl_xor_sync(0xffffffffu, v, o);
  }
  if (lanes <= 32) return v;
  const int warps_per_row = lanes / 32;
  const int warp = threadIdx.x / 32;
  const int row_first_warp = warp - (warp % warps_per_row);
  __syncwarp();
  if ((threadIdx.x & 31) == 0) scratch[warp] = v;
  __syncthreads();
  float total = 0.f;
  for (int i = 0; i < warps_per_row; ++i) total += scratch[row_first_warp + i];
  __syncthreads();
  return total;
}

__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ r,
                                   const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y,
                                   __nv_bfloat16* __restrict__ s_out, float* __restrict__ rstd_out, int rows, int d,
                                   float eps) {
  __shared__ float scratch[32];
  const int lanes = d / 8;
  const int rows_per_block = blockDim.x / lanes;
  const int local_row = threadIdx.x / lanes;
  const int col = (threadIdx.x % lanes) * 8;
  const Vec8 wv = load8(w + col);
  for (int base = blockIdx.x * rows_per_block; base < rows; base += gridDim.x * rows_per_block) {
    const int row = base + local_row;
    const bool live = row < rows;
    Vec8 s = {};
    if (live) {
      s = load8(x + int64_t(row) * d + col);
      if (r != nullptr) {
        Vec8 rv = load8(r + int64_t(row) * d + col);
        #pragma unroll
        for (int i = 0; i < 8; ++i) s.v[i] += rv.v[i];
        // the residual stream is carried in bf16: normalise the rounded sum so that
        // forward and backward see the same s
        #pragma unroll
        for (int i = 0; i < 8; ++i) s.v[i] = __bfloat162float(__float2bfloat16(s.v[i]));
        store8(s_out + int64_t(row) * d + col, s);
      }
    }
    float sq = 0.f;
    #pragma unroll
    for (int i = 0; i < 8; ++i) sq += s.v[i] * s.v[i];
    const float total = row_sum(sq, lanes, scratch);
    const float rstd = rsqrtf(total / float(d) + eps);
    if (live) {
      Vec8 o;
      #pragma unroll
      for (int i = 0; i < 8; ++i) o.v[i] = s.v[i] * rstd * wv.v[i];
      store8(y + int64_t(row) * d + col, o);
      if ((threadIdx.x % lanes) == 0) rstd_out[row] = rstd;
    }
  }
}

__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ s,
                                   const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                                   const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ ds,
                                   float* __restrict__ dw_partial, int rows, int d) {
  __shared__ float scratch[32];
  const int lanes = d / 8;
  const int rows_per_block = blockDim.x / lanes;
  const int local_row = threadIdx.x / lanes;
  const int col = (threadIdx.x % lanes) * 8;
  const Vec8 wv = load8(w + col);
  float dw_acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int base = blockIdx.x * rows_per_block; base < rows; base += gridDim.x * rows_per_block) {
    const int row = base + local_row;
    const bool live = row < rows;
    Vec8 g = {}, sh = {};
    float rs = 0.f;
    if (live) {
      const Vec8 dyv = load8(dy + int64_t(row) * d + col);
      const Vec8 sv = load8(s + int64_t(row) * d + col);
      rs = rstd[row];
      #pragma unroll
      for (int i = 0; i < 8; ++i) {
        sh.v[i] = sv.v[i] * rs;
        g.v[i] = dyv.v[i] * wv.v[i];
        dw_acc[i] += dyv.v[i] * sh.v[i];
      }
    }
    float dot = 0.f;
    #pragma unroll
    for (int i = 0; i < 8; ++i) dot += g.v[i] * sh.v[i];
    const float mean = row_sum(dot, lanes, scratch) / float(d);
    if (live) {
      Vec8 o;
      #pragma unroll
      for (int i = 0; i < 8; ++i) o.v[i] = rs * (g.v[i] - sh.v[i] * mean);
      if (dres != nullptr) {
        const Vec8 rv = load8(dres + int64_t(row) * d + col);
        #pragma unroll
        for (int i = 0; i < 8; ++i) o.v[i] += rv.v[i];
      }
      store8(ds + int64_t(row) * d + col, o);
    }
  }
  // One fp32 partial row per (block, row slot); column_sum_kernel folds them in order.
  float* out = dw_partial + int64_t(blockIdx.x) * rows_per_block * d;
  #pragma unroll
  for (int i = 0; i < 8; ++i) out[int64_t(local_row) * d + col + i] = dw_acc[i];
}

// dw[c] (+)= sum over partial rows p of partial[p, c], in fixed order.
__global__ void column_sum_kernel(const float* __restrict__ partial, int parts, int d, float* __restrict__ dw,
                                  int accumulate) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= d) return;
  float acc = 0.f;
  for (int p = 0; p < parts; ++p) acc += partial[int64_t(p) * d + c];
  dw[c] = accumulate ? dw[c] + acc : acc;
}

int norm_block(int d) {
  const int lanes = d / 8;
  int rows = lanes >= 256 ? 1 : 256 / lanes;
  return lanes * rows;
}

}  // namespace

int rmsnorm_partial_rows(int rows, int d, int num_sms) {
  const int block = norm_block(d);
  const int rows_per_block = block / (d / 8);
  int grid = std::min((rows + rows_per_block - 1) / rows_per_block, 2 * num_sms);
  return grid * rows_per_block;
}

static void check_d(int d) {
  RESIHP_CHECK(d % 8 == 0 && d / 8 <= 1024 && (d / 8 >= 32 ? (d / 8) % 32 == 0 : (32 % (d / 8)) == 0),
               "rmsnorm width ", d, " unsupported (needs d % 8 == 0, d <= 8192, d/8 dividing or divisible by 32)");
}

void rmsnorm_fwd(const void* x, const void* r, const void* w, void* y, void* s_out, float* rstd, int rows, int d,
                 float eps, int num_sms, cudaStream_t st) {
  check_d(d);
  const int block = norm_block(d);
  const int rows_per_block = block / (d / 8);
  const int grid = std::min((rows + rows_per_block - 1) / rows_per_block, 8 * num_sms);
  rmsnorm_fwd_kernel<<<grid, block, 0, st>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(r),
      static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(y), static_cast<__nv_bfloat16*>(s_out), rstd,
      rows, d, eps);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

void rmsnorm_bwd(const void* dy, const void* s, const void* w, const float* rstd, const void* dres, void* ds,
                 float* partial, float* dw, int accumulate, int rows, int d, int num_sms, cudaStream_t st) {
  check_d(d);
  const int block = norm_block(d);
  const int rows_per_block = block / (d / 8);
  const int grid = std::min((rows + rows_per_block - 1) / rows_per_block, 2 * num_sms);
  rmsnorm_bwd_kernel<<<grid, block, 0, st>>>(
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(s),
      static_cast<const __nv_bfloat16*>(w), rstd, static_cast<const __nv_bfloat16*>(dres),
      static_cast<__nv_bfloat16*>(ds), partial, rows, d);
  RESIHP_CUDA_CHECK(cudaGetLastError());
  column_sum_kernel<<<(d + 255) / 256, 256, 0, st>>>(partial, grid * rows_per_block, d, dw, accumulate);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

}  // namespace resihp

// ---- allocation-free entry point (declared in no_alloc.h) ------------------------------
#include <mutex>

#include "no_alloc.h"

// Scratch of the allocation-free entry point: the per-(block, row slot) fp32 partial
// sums of the weight gradient, one array per device that loads this library.
static __device__ __align__(256) float g_rmsnorm_bwd_scratch[RESIHP_NOALLOC_SCRATCH_FLOATS];

namespace {

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mutex;

// Device address of the scratch array on the current device, looked up once per device
// with that device current (host code only sees a stand-in for the symbol).
cudaError_t noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_rmsnorm_bwd_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

void forget_scratch(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  g_scratch_ptr[dev] = nullptr;
}

bool width_supported(int d) {
  if (d <= 0 || d % 8 != 0 || d / 8 > 1024) return false;
  const int lanes = d / 8;
  return lanes >= 32 ? lanes % 32 == 0 : 32 % lanes == 0;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int resihp_rmsnorm_bwd_noalloc(
    const void* dy, const void* s, const void* w, const float* rstd, const void* dres, void* ds, float* dw,
    int accumulate, int rows, int d, cudaStream_t stream) {
  using namespace resihp;
  if (dy == nullptr || s == nullptr || w == nullptr || rstd == nullptr || ds == nullptr || dw == nullptr || rows < 1 ||
      !width_supported(d))
    return RESIHP_NOALLOC_BAD_ARGUMENT;
  // An error left by an earlier, unrelated call stays with its owner: report it as such
  // without reading (and so clearing) it, and launch nothing.
  if (cudaPeekAtLastError() != cudaSuccess) return RESIHP_NOALLOC_PENDING_ERROR;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RESIHP_NOALLOC_CUDA_ERROR;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return RESIHP_NOALLOC_CUDA_ERROR;
  // Same launch shape as the allocating entry point (rmsnorm_bwd), so results agree.
  const int block = norm_block(d);
  const int rows_per_block = block / (d / 8);
  const int grid = std::min((rows + rows_per_block - 1) / rows_per_block, 2 * sms);
  const long long need = static_cast<long long>(grid) * rows_per_block * d;
  if (need > RESIHP_NOALLOC_SCRATCH_FLOATS) return RESIHP_NOALLOC_TOO_LARGE;
  float* partial = nullptr;
  if (noalloc_scratch(&partial) != cudaSuccess) return RESIHP_NOALLOC_CUDA_ERROR;
  rmsnorm_bwd_kernel<<<grid, block, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(s),
      static_cast<const __nv_bfloat16*>(w), rstd, static_cast<const __nv_bfloat16*>(dres),
      static_cast<__nv_bfloat16*>(ds), partial, rows, d);
  if (cudaGetLastError() != cudaSuccess) return RESIHP_NOALLOC_CUDA_ERROR;
  column_sum_kernel<<<(d + 255) / 256, 256, 0, stream>>>(partial, grid * rows_per_block, d, dw, accumulate);
  if (cudaGetLastError() != cudaSuccess) return RESIHP_NOALLOC_CUDA_ERROR;
  return RESIHP_NOALLOC_OK;
}

extern "C" __attribute__((visibility("default"))) void resihp_noalloc_forget_device(int device) {
  forget_scratch(device);
}

extern "C" __attribute__((visibility("default"))) const char* resihp_noalloc_strerror(int code) {
  switch (code) {
    case RESIHP_NOALLOC_OK: return "ok";
    case RESIHP_NOALLOC_BAD_ARGUMENT: return "bad argument: null pointer, rows < 1, or unsupported width d";
    case RESIHP_NOALLOC_TOO_LARGE:
      return "scratch need exceeds the built-in 16 MiB (RESIHP_NOALLOC_SCRATCH_FLOATS) scratch array";
    case RESIHP_NOALLOC_CUDA_ERROR: return "a CUDA runtime call or kernel launch failed";
    case RESIHP_NOALLOC_PENDING_ERROR:
      return "an earlier CUDA error was pending on this thread; nothing was launched and the error is left in place";
    default: return "unknown error code";
  }
}
