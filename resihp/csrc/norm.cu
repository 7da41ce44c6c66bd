// RMSNorm forward/backward (bf16 activations, fp32 statistics), with the residual add of
// a pre-norm block fused in (the Llama counterpart of the reference's ``F.layer_norm``
// calls, resihp/parallel/tp.py:262,264,268, and their residual adds):
//
//   forward   s = x (+ r);   y = s * rstd * w,   rstd = 1 / sqrt(mean(s^2) + eps)
//   backward  g = dy * w;    ds = rstd * (g - s_hat * mean(g * s_hat)) (+ dres),
//             dw += sum_rows dy * s_hat                  (s_hat = s * rstd)
//
// Widths 256-2048 run warp-per-row kernels: a warp owns a row, each lane 8-column
// vectors of it (the backward keeps the row in packed registers between its two passes;
// the optional streaming backward reads it again instead). Other widths run the general
// kernels, where one row is spread over d/8 threads, each holding one 16-byte vector (8
// bf16), and several rows share a block so that a block has >= 256 threads. The weight
// gradient is reduced deterministically: every block of a fixed-size persistent grid
// writes one fp32 partial row, and a second kernel sums the partials in block order.
#include <algorithm>
#include <cstdlib>
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
  pdl_enter();
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
  pdl_enter();
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
  pdl_enter();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= d) return;
  float acc = 0.f;
  for (int p = 0; p < parts; ++p) acc += partial[int64_t(p) * d + c];
  dw[c] = accumulate ? dw[c] + acc : acc;
}

// ---- warp-per-row variants for d = 256 * VPL (VPL = 1, 2, 4, 8) ------------------------
// A warp owns a whole row: lane l holds the 16-byte vectors at columns (32 j + l) * 8,
// j < VPL (each j one coalesced 512-byte warp access), the row statistics are warp
// shuffles (no block barrier per row), and every lane has 2 VPL loads in flight. The
// weight-gradient partials of a block's eight warps are added in warp order in shared
// memory, one fp32 partial row per block.

__device__ __forceinline__ float warp_sum(float v) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int kNormWarps = 8;


template <int VPL>
__global__ void __launch_bounds__(32 * kNormWarps)
    rmsnorm_fwd_warp_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ r,
                            const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y,
                            __nv_bfloat16* __restrict__ s_out, float* __restrict__ rstd_out, int rows, float eps) {
  pdl_enter();
  constexpr int D = 256 * VPL;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * kNormWarps + (threadIdx.x >> 5); row < rows; row += gridDim.x * kNormWarps) {
    const int64_t base = int64_t(row) * D;
    Vec8 sv[VPL];
    #pragma unroll
    for (int j = 0; j < VPL; ++j) sv[j] = load8(x + base + (32 * j + lane) * 8);
    if (r != nullptr) {
      #pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const Vec8 rv = load8(r + base + (32 * j + lane) * 8);
        #pragma unroll
        for (int i = 0; i < 8; ++i) sv[j].v[i] = __bfloat162float(__float2bfloat16(sv[j].v[i] + rv.v[i]));
        store8(s_out + base + (32 * j + lane) * 8, sv[j]);
      }
    }
    float sq = 0.f;
    #pragma unroll
    for (int j = 0; j < VPL; ++j)
      #pragma unroll
      for (int i = 0; i < 8; ++i) sq += sv[j].v[i] * sv[j].v[i];
    const float rstd = rsqrtf(warp_sum(sq) / float(D) + eps);
    #pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const Vec8 wv = load8(w + (32 * j + lane) * 8);
      Vec8 o;
      #pragma unroll
      for (int i = 0; i < 8; ++i) o.v[i] = sv[j].v[i] * rstd * wv.v[i];
      store8(y + base + (32 * j + lane) * 8, o);
    }
    if (lane == 0) rstd_out[row] = rstd;
  }
}

template <int VPL>
__global__ void __launch_bounds__(32 * kNormWarps)
    rmsnorm_bwd_warp_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ s,
                            const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                            const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ ds,
                            float* __restrict__ dw_partial, int rows) {
  pdl_enter();
  constexpr int D = 256 * VPL;
  extern __shared__ float4 dw_smem4[];  // [kNormWarps][D / 4]: each warp's running dw row
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float4* mine = dw_smem4 + warp * (D / 4);
  #pragma unroll
  for (int j = 0; j < VPL; ++j) {
    mine[(32 * j + lane) * 2] = make_float4(0.f, 0.f, 0.f, 0.f);
    mine[(32 * j + lane) * 2 + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  uint4 wr[VPL];  // this lane's weights, packed, for every row
  #pragma unroll
  for (int j = 0; j < VPL; ++j) wr[j] = *reinterpret_cast<const uint4*>(w + (32 * j + lane) * 8);
  const int step = gridDim.x * kNormWarps;
  for (int row = blockIdx.x * kNormWarps + warp; row < rows; row += step) {
    const int64_t base = int64_t(row) * D;
    // the warp's next row heads for L2 while this one is loaded and reduced
    if (lane == 0 && row + step < rows) {
      const int64_t nb = base + int64_t(step) * D;
      l2_prefetch_bulk(dy + nb, D * 2);
      l2_prefetch_bulk(s + nb, D * 2);
      if (dres != nullptr) l2_prefetch_bulk(dres + nb, D * 2);
    }
    const float rs = rstd[row];
    // every load of the row in flight at once, kept packed (bf16) through the reduction
    uint4 dyr[VPL], sr[VPL], rr[VPL];
    #pragma unroll
    for (int j = 0; j < VPL; ++j) {
      dyr[j] = *reinterpret_cast<const uint4*>(dy + base + (32 * j + lane) * 8);
      sr[j] = *reinterpret_cast<const uint4*>(s + base + (32 * j + lane) * 8);
      if (dres != nullptr) rr[j] = *reinterpret_cast<const uint4*>(dres + base + (32 * j + lane) * 8);
    }
    float dot = 0.f;
    #pragma unroll
    for (int j = 0; j < VPL; ++j) {
      asm volatile("" : "+r"(wr[j].x), "+r"(wr[j].y), "+r"(wr[j].z), "+r"(wr[j].w));
      const Vec8 dyv = load8(reinterpret_cast<const __nv_bfloat16*>(&dyr[j]));
      const Vec8 svv = load8(reinterpret_cast<const __nv_bfloat16*>(&sr[j]));
      const Vec8 wv = load8(reinterpret_cast<const __nv_bfloat16*>(&wr[j]));
      #pragma unroll
      for (int i = 0; i < 8; ++i) dot += dyv.v[i] * wv.v[i] * (svv.v[i] * rs);
    }
    const float mean = warp_sum(dot) / float(D);
    #pragma unroll
    for (int j = 0; j < VPL; ++j) {
      // unpack again rather than keep the unpacked floats of the first loop alive
      // (register pressure): the empty asm hides that the values are unchanged
      asm volatile("" : "+r"(dyr[j].x), "+r"(dyr[j].y), "+r"(dyr[j].z), "+r"(dyr[j].w));
      asm volatile("" : "+r"(sr[j].x), "+r"(sr[j].y), "+r"(sr[j].z), "+r"(sr[j].w));
      asm volatile("" : "+r"(wr[j].x), "+r"(wr[j].y), "+r"(wr[j].z), "+r"(wr[j].w));
      const Vec8 dyv = load8(reinterpret_cast<const __nv_bfloat16*>(&dyr[j]));
      const Vec8 svv = load8(reinterpret_cast<const __nv_bfloat16*>(&sr[j]));
      const Vec8 wv = load8(reinterpret_cast<const __nv_bfloat16*>(&wr[j]));
      Vec8 o;
      float sh[8];
      #pragma unroll
      for (int i = 0; i < 8; ++i) {
        sh[i] = svv.v[i] * rs;
        o.v[i] = rs * (dyv.v[i] * wv.v[i] - sh[i] * mean);
      }
      if (dres != nullptr) {
        const Vec8 rv = load8(reinterpret_cast<const __nv_bfloat16*>(&rr[j]));
        #pragma unroll
        for (int i = 0; i < 8; ++i) o.v[i] += rv.v[i];
      }
      store8(ds + base + (32 * j + lane) * 8, o);
      float4 a = mine[(32 * j + lane) * 2], b = mine[(32 * j + lane) * 2 + 1];
      a.x += dyv.v[0] * sh[0]; a.y += dyv.v[1] * sh[1]; a.z += dyv.v[2] * sh[2]; a.w += dyv.v[3] * sh[3];
      b.x += dyv.v[4] * sh[4]; b.y += dyv.v[5] * sh[5]; b.z += dyv.v[6] * sh[6]; b.w += dyv.v[7] * sh[7];
      mine[(32 * j + lane) * 2] = a;
      mine[(32 * j + lane) * 2 + 1] = b;
    }
  }
  __syncthreads();
  const float* dw_smem = reinterpret_cast<const float*>(dw_smem4);
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
    #pragma unroll
    for (int q = 0; q < kNormWarps; ++q) acc += dw_smem[q * D + c];
    dw_partial[int64_t(blockIdx.x) * D + c] = acc;
  }
}

// The same backward in a streaming form (RESIHP_NORM_STREAM=1, experimental): no row
// stays in registers between the two passes -- the second pass reads dy and s again (L2
// hits: the row was just read) -- so a thread needs ~80 registers instead of ~250 and
// three CTAs share an SM: 24 warps, about one row each at the 1.3B shapes, all in flight
// at once instead of a third of them. Same per-element arithmetic and the same order of
// the row reduction as the register kernel (ds is identical); dw goes through per-warp
// shared-memory rows as there, over this kernel's grid.
constexpr int kStreamCtasPerSm = 3;

template <int VPL>
__global__ void __launch_bounds__(32 * kNormWarps, kStreamCtasPerSm)
    rmsnorm_bwd_stream_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ s,
                              const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                              const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ ds,
                              float* __restrict__ dw_partial, int rows) {
  pdl_enter();
  constexpr int D = 256 * VPL;
  extern __shared__ float4 dw_smem4[];  // [kNormWarps][D / 4]: each warp's running dw row
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float4* mine = dw_smem4 + warp * (D / 4);
  #pragma unroll
  for (int j = 0; j < VPL; ++j) {
    mine[(32 * j + lane) * 2] = make_float4(0.f, 0.f, 0.f, 0.f);
    mine[(32 * j + lane) * 2 + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int row = blockIdx.x * kNormWarps + warp; row < rows; row += gridDim.x * kNormWarps) {
    const int64_t base = int64_t(row) * D;
    const float rs = rstd[row];
    float dot = 0.f;
    #pragma unroll 2
    for (int j = 0; j < VPL; ++j) {
      const int col = (32 * j + lane) * 8;
      const Vec8 dyv = load8(dy + base + col);
      const Vec8 svv = load8(s + base + col);
      const Vec8 wv = load8(w + col);
      #pragma unroll
      for (int i = 0; i < 8; ++i) dot += dyv.v[i] * wv.v[i] * (svv.v[i] * rs);
    }
    const float mean = warp_sum(dot) / float(D);
    #pragma unroll 2
    for (int j = 0; j < VPL; ++j) {
      const int col = (32 * j + lane) * 8;
      const Vec8 dyv = load8(dy + base + col);
      const Vec8 svv = load8(s + base + col);
      const Vec8 wv = load8(w + col);
      Vec8 o;
      float sh[8];
      #pragma unroll
      for (int i = 0; i < 8; ++i) {
        sh[i] = svv.v[i] * rs;
        o.v[i] = rs * (dyv.v[i] * wv.v[i] - sh[i] * mean);
      }
      if (dres != nullptr) {
        const Vec8 rv = load8(dres + base + col);
        #pragma unroll
        for (int i = 0; i < 8; ++i) o.v[i] += rv.v[i];
      }
      store8(ds + base + col, o);
      float4 a = mine[(32 * j + lane) * 2], b = mine[(32 * j + lane) * 2 + 1];
      a.x += dyv.v[0] * sh[0]; a.y += dyv.v[1] * sh[1]; a.z += dyv.v[2] * sh[2]; a.w += dyv.v[3] * sh[3];
      b.x += dyv.v[4] * sh[4]; b.y += dyv.v[5] * sh[5]; b.z += dyv.v[6] * sh[6]; b.w += dyv.v[7] * sh[7];
      mine[(32 * j + lane) * 2] = a;
      mine[(32 * j + lane) * 2 + 1] = b;
    }
  }
  __syncthreads();
  const float* dw_smem = reinterpret_cast<const float*>(dw_smem4);
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
    #pragma unroll
    for (int q = 0; q < kNormWarps; ++q) acc += dw_smem[q * D + c];
    dw_partial[int64_t(blockIdx.x) * D + c] = acc;
  }
}

// dw[c] (+)= sum over partial rows of partial[p, c] in a fixed order: block (32 columns
// x 8 groups); group g sums rows g, g+8, g+16, ... in turn, then the 8 group sums are
// added in group order. Used with the warp-per-row backward (fewer, wider blocks than
// column_sum_kernel's one thread per column would keep busy).
__global__ void column_sum_wide_kernel(const float* __restrict__ partial, int parts, int d, float* __restrict__ dw,
                                       int accumulate) {
  pdl_enter();
  __shared__ float sums[8][33];
  const int cl = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + cl;
  float acc = 0.f;
  if (c < d)
    for (int p = grp; p < parts; p += 8) acc += partial[int64_t(p) * d + c];
  sums[grp][cl] = acc;
  __syncthreads();
  if (grp == 0 && c < d) {
    float tot = 0.f;
    #pragma unroll
    for (int q = 0; q < 8; ++q) tot += sums[q][cl];
    dw[c] = accumulate ? dw[c] + tot : tot;
  }
}

// VPL of the warp-per-row kernels for width d, or 0 for the general kernels.
int norm_vpl(int d) {
  return (d == 256 || d == 512 || d == 1024 || d == 2048) ? d / 256 : 0;
}

// RESIHP_NORM_STREAM=1 selects the streaming backward (experimental).
bool norm_stream() {
  static const bool on = [] {
    const char* e = std::getenv("RESIHP_NORM_STREAM");
    return e != nullptr && e[0] == '1';
  }();
  return on;
}

int warp_norm_grid(int rows, int num_sms) {
  return std::max(1, std::min((rows + kNormWarps - 1) / kNormWarps, num_sms));
}

// Grid of the warp-per-row backward: one CTA per SM, or (streaming) kStreamCtasPerSm.
int bwd_norm_grid(int rows, int num_sms) {
  return norm_stream() ? std::max(1, std::min((rows + kNormWarps - 1) / kNormWarps, kStreamCtasPerSm * num_sms))
                       : warp_norm_grid(rows, num_sms);
}

int norm_block(int d) {
  const int lanes = d / 8;
  int rows = lanes >= 256 ? 1 : 256 / lanes;
  return lanes * rows;
}

}  // namespace

int rmsnorm_partial_rows(int rows, int d, int num_sms) {
  if (norm_vpl(d) != 0) return bwd_norm_grid(rows, num_sms);
  const int block = norm_block(d);
  const int rows_per_block = block / (d / 8);
  int grid = std::min((rows + rows_per_block - 1) / rows_per_block, 2 * num_sms);
  return grid * rows_per_block;
}

namespace {

template <int VPL>
void launch_bwd_warp(const void* dy, const void* s, const void* w, const float* rstd, const void* dres, void* ds,
                     float* partial, int rows, int grid, cudaStream_t st) {
  constexpr int smem = kNormWarps * 256 * VPL * int(sizeof(float));
  auto kernel = norm_stream() ? rmsnorm_bwd_stream_kernel<VPL> : rmsnorm_bwd_warp_kernel<VPL>;
  if (smem > 48 * 1024) (void)cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  launch_pdl(kernel, grid, 32 * kNormWarps, smem, st,
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(s),
      static_cast<const __nv_bfloat16*>(w), rstd, static_cast<const __nv_bfloat16*>(dres),
      static_cast<__nv_bfloat16*>(ds), partial, rows);
}

}  // namespace

// The backward's two launches into a caller-provided ``partial`` buffer of
// rmsnorm_partial_rows(rows, d, num_sms) x d floats (shared by both entry points).
cudaError_t rmsnorm_bwd_launch(const void* dy, const void* s, const void* w, const float* rstd, const void* dres,
                               void* ds, float* partial, float* dw, int accumulate, int rows, int d, int num_sms,
                               cudaStream_t st) {
  const int vpl = norm_vpl(d);
  if (vpl != 0) {
    const int grid = bwd_norm_grid(rows, num_sms);
    switch (vpl) {
      case 1: launch_bwd_warp<1>(dy, s, w, rstd, dres, ds, partial, rows, grid, st); break;
      case 2: launch_bwd_warp<2>(dy, s, w, rstd, dres, ds, partial, rows, grid, st); break;
      case 4: launch_bwd_warp<4>(dy, s, w, rstd, dres, ds, partial, rows, grid, st); break;
      default: launch_bwd_warp<8>(dy, s, w, rstd, dres, ds, partial, rows, grid, st); break;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    launch_pdl(column_sum_wide_kernel, (d + 31) / 32, 256, 0, st, partial, grid, d, dw, accumulate);
    return cudaGetLastError();
  }
  const int block = norm_block(d);
  const int rows_per_block = block / (d / 8);
  const int grid = std::min((rows + rows_per_block - 1) / rows_per_block, 2 * num_sms);
  launch_pdl(rmsnorm_bwd_kernel, grid, block, 0, st,
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(s),
      static_cast<const __nv_bfloat16*>(w), rstd, static_cast<const __nv_bfloat16*>(dres),
      static_cast<__nv_bfloat16*>(ds), partial, rows, d);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  launch_pdl(column_sum_kernel, (d + 255) / 256, 256, 0, st, partial, grid * rows_per_block, d, dw, accumulate);
  return cudaGetLastError();
}

static void check_d(int d) {
  RESIHP_CHECK(d % 8 == 0 && d / 8 <= 1024 && (d / 8 >= 32 ? (d / 8) % 32 == 0 : (32 % (d / 8)) == 0),
               "rmsnorm width ", d, " unsupported (needs d % 8 == 0, d <= 8192, d/8 dividing or divisible by 32)");
}

void rmsnorm_fwd(const void* x, const void* r, const void* w, void* y, void* s_out, float* rstd, int rows, int d,
                 float eps, int num_sms, cudaStream_t st) {
  check_d(d);
  const int vpl = norm_vpl(d);
  if (vpl != 0) {
    const int grid = std::max(1, std::min((rows + kNormWarps - 1) / kNormWarps, 8 * num_sms));
    const auto* xb = static_cast<const __nv_bfloat16*>(x);
    const auto* rb = static_cast<const __nv_bfloat16*>(r);
    const auto* wb = static_cast<const __nv_bfloat16*>(w);
    auto* yb = static_cast<__nv_bfloat16*>(y);
    auto* sb = static_cast<__nv_bfloat16*>(s_out);
    switch (vpl) {
      case 1: launch_pdl(rmsnorm_fwd_warp_kernel<1>, grid, 32 * kNormWarps, 0, st, xb, rb, wb, yb, sb, rstd, rows, eps); break;
      case 2: launch_pdl(rmsnorm_fwd_warp_kernel<2>, grid, 32 * kNormWarps, 0, st, xb, rb, wb, yb, sb, rstd, rows, eps); break;
      case 4: launch_pdl(rmsnorm_fwd_warp_kernel<4>, grid, 32 * kNormWarps, 0, st, xb, rb, wb, yb, sb, rstd, rows, eps); break;
      default: launch_pdl(rmsnorm_fwd_warp_kernel<8>, grid, 32 * kNormWarps, 0, st, xb, rb, wb, yb, sb, rstd, rows, eps); break;
    }
    RESIHP_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const int block = norm_block(d);
  const int rows_per_block = block / (d / 8);
  const int grid = std::min((rows + rows_per_block - 1) / rows_per_block, 8 * num_sms);
  launch_pdl(rmsnorm_fwd_kernel, grid, block, 0, st,
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(r),
      static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(y), static_cast<__nv_bfloat16*>(s_out), rstd,
      rows, d, eps);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

void rmsnorm_bwd(const void* dy, const void* s, const void* w, const float* rstd, const void* dres, void* ds,
                 float* partial, float* dw, int accumulate, int rows, int d, int num_sms, cudaStream_t st) {
  check_d(d);
  RESIHP_CUDA_CHECK(rmsnorm_bwd_launch(dy, s, w, rstd, dres, ds, partial, dw, accumulate, rows, d, num_sms, st));
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
  // The same launches as the allocating entry point (rmsnorm_bwd), so results agree.
  const long long need = static_cast<long long>(rmsnorm_partial_rows(rows, d, sms)) * d;
  if (need > RESIHP_NOALLOC_SCRATCH_FLOATS) return RESIHP_NOALLOC_TOO_LARGE;
  float* partial = nullptr;
  if (noalloc_scratch(&partial) != cudaSuccess) return RESIHP_NOALLOC_CUDA_ERROR;
  if (rmsnorm_bwd_launch(dy, s, w, rstd, dres, ds, partial, dw, accumulate, rows, d, sms, stream) != cudaSuccess)
    return RESIHP_NOALLOC_CUDA_ERROR;
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
