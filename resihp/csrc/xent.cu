// Vocab-parallel cross-entropy over bf16 logits, so full logits are never gathered
// (reference: ``F.cross_entropy`` resihp/reference.py:41-50 over logits all-gathered by
// ``_GatherLastDim`` resihp/parallel/tp.py:92-110,272-273).
//
// Pass 1 (xent_stats): per row of this rank's vocab shard, the shard max, the sum of
// exp(x - max) and the target logit when the label falls in the shard. Across TP ranks
// the three small [rows] vectors are combined (max-all-reduce, rescaled sum, sum) into
// the log-sum-exp, without ever materialising the [rows, V] logits.
// Pass 2 (xent_grad): d logits = (softmax - onehot) * scale, written over the logits.
// Rows whose label is negative are ignored (zero loss, zero gradient).
#include <cuda_bf16.h>

#include "common.cuh"
#include "launch.h"

namespace resihp {

namespace {

constexpr int kXentThreads = 512;

__device__ __forceinline__ void merge(float& m, float& s, float m2, float s2) {
  if (m2 > m) {
    s = s * __expf(m - m2) + s2;
    m = m2;
  } else if (m2 != -INFINITY) {
    s = s + s2 * __expf(m2 - m);
  }
}

__global__ void xent_stats_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld,
                                  const int64_t* __restrict__ labels, float* __restrict__ stats, int rows, int v,
                                  int64_t start) {
  pdl_enter();
  __shared__ float sm_m[kXentThreads / 32], sm_s[kXentThreads / 32];
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + int64_t(row) * ld;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x * 8; c < v; c += blockDim.x * 8) {
    uint4 raw = *reinterpret_cast<const uint4*>(x + c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float vals[8];
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      vals[2 * i] = f.x;
      vals[2 * i + 1] = f.y;
    }
    float lm = vals[0];
    #pragma unroll
    for (int i = 1; i < 8; ++i) lm = fmaxf(lm, vals[i]);
    float ls = 0.f;
    #pragma unroll
    for (int i = 0; i < 8; ++i) ls += __expf(vals[i] - lm);
    merge(m, s, lm, ls);
  }
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge(m, s, m2, s2);
  }
  const int warp = threadIdx.x / 32;
  if ((threadIdx.x & 31) == 0) {
    sm_m[warp] = m;
    sm_s[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = sm_m[0], ss = sm_s[0];
    for (int w = 1; w < int(blockDim.x / 32); ++w) merge(mm, ss, sm_m[w], sm_s[w]);
    const int64_t label = labels[row];
    const int64_t local = label - start;
    const bool mine = label >= 0 && local >= 0 && local < v;
    stats[3 * row + 0] = mm;
    stats[3 * row + 1] = ss;
    stats[3 * row + 2] = mine ? __bfloat162float(x[local]) : 0.f;
  }
}

__global__ void xent_grad_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld, const int64_t* __restrict__ labels,
                                 const float* __restrict__ lse, const float* __restrict__ scale, int rows, int v,
                                 int64_t start) {
  pdl_enter();
  const int row = blockIdx.x;
  __nv_bfloat16* x = logits + int64_t(row) * ld;
  const int64_t label = labels[row];
  const float l = lse[row];
  const float sc = label < 0 ? 0.f : scale[0];
  const int64_t local = label - start;
  for (int c = threadIdx.x * 8; c < v; c += blockDim.x * 8) {
    uint4 raw = *reinterpret_cast<const uint4*>(x + c);
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
    uint32_t out[4];
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      float a = __expf(f.x - l), b = __expf(f.y - l);
      if (c + 2 * i == local) a -= 1.f;
      if (c + 2 * i + 1 == local) b -= 1.f;
      out[i] = pack_bf16(a * sc, b * sc);
    }
    *reinterpret_cast<uint4*>(x + c) = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

}  // namespace

void xent_stats(const void* logits, int64_t ld, const int64_t* labels, float* stats, int rows, int v, int64_t start,
                cudaStream_t st) {
  RESIHP_CHECK(v % 8 == 0 && ld % 8 == 0, "cross-entropy vocab shard must be a multiple of 8");
  launch_pdl(xent_stats_kernel, rows, kXentThreads, 0, st, static_cast<const __nv_bfloat16*>(logits), ld, labels, stats, rows,
                                                   v, start);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

void xent_grad(void* logits, int64_t ld, const int64_t* labels, const float* lse, const float* scale, int rows, int v,
               int64_t start, cudaStream_t st) {
  RESIHP_CHECK(v % 8 == 0 && ld % 8 == 0, "cross-entropy vocab shard must be a multiple of 8");
  launch_pdl(xent_grad_kernel, rows, 256, 0, st, static_cast<__nv_bfloat16*>(logits), ld, labels, lse, scale, rows, v, start);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

}  // namespace resihp
