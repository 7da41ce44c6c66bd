// Memory-bound kernels of the Llama block and the optimizer (reference counterparts:
// ``F.gelu`` MLP activation resihp/parallel/tp.py:247, ``torch.optim.AdamW``
// resihp/reference.py:29-38 stepped at resihp/parallel/pp.py:451, vocab-parallel
// embedding resihp/parallel/tp.py:222-228):
//   * RoPE (rotate-half / GPT-NeoX pairing) applied in place to the Q and K heads of
//     the fused QKV activation, forward and backward (backward rotates by -theta);
//   * SwiGLU  h = silu(g) * u  over the fused [g | u] projection, forward and backward;
//   * AdamW over flat fp32 buffers, writing the bf16 working copy in the same pass;
//   * vocab-parallel embedding lookup, and its deterministic backward (runs of equal
//     token ids, pre-sorted, are summed in order by one block each).
#include <cuda_bf16.h>

#include "common.cuh"
#include "launch.h"

namespace resihp {

namespace {

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

// qkv: [rows, (hq + 2*hkv) * hd] bf16; row t has sequence position t % seq.
// cs: [seq, hd/2, 2] fp32 = (cos, sin) of position * inv_freq[i].
// Each thread rotates one (i, i + hd/2) pair of one Q or K head.
__global__ void rope_kernel(__nv_bfloat16* __restrict__ qkv, const float2* __restrict__ cs, int rows, int seq,
                            int heads_qk, int hd, int64_t row_stride, int pos_offset, float sign) {
  pdl_enter();
  const int half = hd / 2;
  const int64_t total = int64_t(rows) * heads_qk * half;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int p = int(i % half);
    const int64_t rh = i / half;
    const int h = int(rh % heads_qk);
    const int64_t row = rh / heads_qk;
    const int pos = int((row + pos_offset) % seq);
    const float2 c = cs[int64_t(pos) * half + p];
    __nv_bfloat16* base = qkv + row * row_stride + int64_t(h) * hd;
    const float x1 = bf(base[p]);
    const float x2 = bf(base[p + half]);
    const float sn = sign * c.y;
    base[p] = __float2bfloat16(x1 * c.x - x2 * sn);
    base[p + half] = __float2bfloat16(x2 * c.x + x1 * sn);
  }
}

// Rotates eight (x1, x2) pairs held as two 16-byte vectors; c4 points at the pairs'
// (cos, sin) values, two pairs per float4.
__device__ __forceinline__ void rope8(uint4& r1, uint4& r2, const float4* __restrict__ c4, float sign) {
  const __nv_bfloat162* x1 = reinterpret_cast<const __nv_bfloat162*>(&r1);
  const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&r2);
  uint32_t o1[4], o2[4];
  #pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 c = c4[q];  // (cos, sin) of pairs 2q, 2q+1
    const float2 a = __bfloat1622float2(x1[q]), bb = __bfloat1622float2(x2[q]);
    const float s0 = sign * c.y, s1 = sign * c.w;
    o1[q] = pack_bf16(a.x * c.x - bb.x * s0, a.y * c.z - bb.y * s1);
    o2[q] = pack_bf16(bb.x * c.x + a.x * s0, bb.y * c.z + a.y * s1);
  }
  r1 = make_uint4(o1[0], o1[1], o1[2], o1[3]);
  r2 = make_uint4(o2[0], o2[1], o2[2], o2[3]);
}

// Vector form (hd % 16 == 0, 16-byte aligned rows): one thread rotates eight pairs
// (p..p+7, p+hd/2..p+hd/2+7) with two 16-byte loads and stores; a block walks rows
// (grid-stride) two at a time, so each thread has both rows' loads in flight before it
// computes, and its threads the rows' Q/K head vectors (no 64-bit division per element).
__global__ void rope_vec_kernel(__nv_bfloat16* __restrict__ qkv, const float2* __restrict__ cs, int rows, int seq,
                                int heads_qk, int hd, int64_t row_stride, int pos_offset, float sign) {
  pdl_enter();
  const int half = hd / 2, vph = half / 8;
  const int per_row = heads_qk * vph;
  for (int row = blockIdx.x; row < rows; row += 2 * gridDim.x) {
    const int row2 = row + gridDim.x;
    const bool two = row2 < rows;
    const float4* c4a = reinterpret_cast<const float4*>(cs + int64_t((row + pos_offset) % seq) * half);
    const float4* c4b = reinterpret_cast<const float4*>(cs + int64_t((row2 + pos_offset) % seq) * half);
    __nv_bfloat16* ra = qkv + int64_t(row) * row_stride;
    __nv_bfloat16* rb = qkv + int64_t(row2) * row_stride;
    for (int j = threadIdx.x; j < per_row; j += blockDim.x) {
      const int h = j / vph, v = j - h * vph;
      const int off = h * hd + v * 8;
      uint4 a1 = *reinterpret_cast<const uint4*>(ra + off);
      uint4 a2 = *reinterpret_cast<const uint4*>(ra + off + half);
      uint4 b1, b2;
      if (two) {
        b1 = *reinterpret_cast<const uint4*>(rb + off);
        b2 = *reinterpret_cast<const uint4*>(rb + off + half);
      }
      rope8(a1, a2, c4a + v * 4, sign);
      *reinterpret_cast<uint4*>(ra + off) = a1;
      *reinterpret_cast<uint4*>(ra + off + half) = a2;
      if (two) {
        rope8(b1, b2, c4b + v * 4, sign);
        *reinterpret_cast<uint4*>(rb + off) = b1;
        *reinterpret_cast<uint4*>(rb + off + half) = b2;
      }
    }
  }
}

// The fast (approximate) division: an IEEE divide per element made the SwiGLU forward
// arithmetic-bound (8 sigmoids per 48 bytes moved); for x -> -inf the denominator
// overflows to inf and the quotient is 0, the limit.
__device__ __forceinline__ float sigmoid(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// gu: [rows, 2F] = [g | u];  h: [rows, F]
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ h, int rows,
                                  int f) {
  pdl_enter();
  const int64_t total = int64_t(rows) * f / 2;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t row = (2 * i) / f;
    const int col = int((2 * i) % f);
    const __nv_bfloat162 g = *reinterpret_cast<const __nv_bfloat162*>(gu + row * 2 * f + col);
    const __nv_bfloat162 u = *reinterpret_cast<const __nv_bfloat162*>(gu + row * 2 * f + f + col);
    const float2 gf = __bfloat1622float2(g), uf = __bfloat1622float2(u);
    const float a = gf.x * sigmoid(gf.x) * uf.x;
    const float b = gf.y * sigmoid(gf.y) * uf.y;
    *reinterpret_cast<uint32_t*>(h + row * f + col) = pack_bf16(a, b);
  }
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu, const __nv_bfloat16* __restrict__ dh,
                                  __nv_bfloat16* __restrict__ dgu, int rows, int f) {
  pdl_enter();
  const int64_t total = int64_t(rows) * f / 2;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t row = (2 * i) / f;
    const int col = int((2 * i) % f);
    const float2 gf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(gu + row * 2 * f + col));
    const float2 uf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(gu + row * 2 * f + f + col));
    const float2 d = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(dh + row * f + col));
    float dg[2], du[2];
    const float g2[2] = {gf.x, gf.y}, u2[2] = {uf.x, uf.y}, d2[2] = {d.x, d.y};
    #pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float s = sigmoid(g2[j]);
      const float silu = g2[j] * s;
      du[j] = d2[j] * silu;
      dg[j] = d2[j] * u2[j] * s * (1.f + g2[j] * (1.f - s));
    }
    *reinterpret_cast<uint32_t*>(dgu + row * 2 * f + col) = pack_bf16(dg[0], dg[1]);
    *reinterpret_cast<uint32_t*>(dgu + row * 2 * f + f + col) = pack_bf16(du[0], du[1]);
  }
}

// Vector forms (f % 8 == 0): one thread per 8 columns of a row, 16-byte accesses, and
// the row / column split is one 32-bit division per 8 elements.
__global__ void swiglu_fwd_vec_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ h, int rows,
                                      int f) {
  pdl_enter();
  const unsigned vpr = unsigned(f) / 8u;
  const unsigned total = unsigned(rows) * vpr;
  const unsigned stride = gridDim.x * blockDim.x;
  // two items per thread and iteration: all four loads are issued before any compute
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += 2 * stride) {
    uint4 gr[2], ur[2];
    int64_t out[2];
    #pragma unroll
    for (int t = 0; t < 2; ++t) {
      const unsigned it = i + t * stride;
      if (t == 0 || it < total) {
        const unsigned row = it / vpr, col = (it - row * vpr) * 8u;
        const __nv_bfloat16* g = gu + int64_t(row) * 2 * f + col;
        gr[t] = *reinterpret_cast<const uint4*>(g);
        ur[t] = *reinterpret_cast<const uint4*>(g + f);
        out[t] = int64_t(row) * f + col;
      }
    }
    #pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (t == 1 && i + stride >= total) break;
      const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gr[t]);
      const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&ur[t]);
      uint32_t o[4];
      #pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 gf = __bfloat1622float2(g2[q]), uf = __bfloat1622float2(u2[q]);
        o[q] = pack_bf16(gf.x * sigmoid(gf.x) * uf.x, gf.y * sigmoid(gf.y) * uf.y);
      }
      *reinterpret_cast<uint4*>(h + out[t]) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

__global__ void swiglu_bwd_vec_kernel(const __nv_bfloat16* __restrict__ gu, const __nv_bfloat16* __restrict__ dh,
                                      __nv_bfloat16* __restrict__ dgu, int rows, int f) {
  pdl_enter();
  const unsigned vpr = unsigned(f) / 8u;
  const unsigned total = unsigned(rows) * vpr;
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const unsigned row = i / vpr, col = (i - row * vpr) * 8u;
    const int64_t gbase = int64_t(row) * 2 * f + col;
    const uint4 gr = *reinterpret_cast<const uint4*>(gu + gbase);
    const uint4 ur = *reinterpret_cast<const uint4*>(gu + gbase + f);
    const uint4 dr = *reinterpret_cast<const uint4*>(dh + int64_t(row) * f + col);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gr);
    const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&ur);
    const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&dr);
    uint32_t og[4], ou[4];
    #pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 gf = __bfloat1622float2(g2[q]), uf = __bfloat1622float2(u2[q]), df = __bfloat1622float2(d2[q]);
      const float sx = sigmoid(gf.x), sy = sigmoid(gf.y);
      og[q] = pack_bf16(df.x * uf.x * sx * (1.f + gf.x * (1.f - sx)), df.y * uf.y * sy * (1.f + gf.y * (1.f - sy)));
      ou[q] = pack_bf16(df.x * gf.x * sx, df.y * gf.y * sy);
    }
    *reinterpret_cast<uint4*>(dgu + gbase) = make_uint4(og[0], og[1], og[2], og[3]);
    *reinterpret_cast<uint4*>(dgu + gbase + f) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
  }
}

// AdamW step over flat fp32 buffers, the torch.optim.AdamW formulation:
//   p *= 1 - lr*wd;  m = m + (1-b1)(g-m);  v = b2 v + (1-b2) g^2
//   p -= (lr / bc1) * m / (sqrt(v) / sqrt(bc2) + eps)
// and the bf16 working copy of p is refreshed in the same pass.
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ p_bf16, int64_t n, AdamWCoef c) {
  pdl_enter();
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    float pi = p[i], mi = m[i], vi = v[i];
    adamw_elem(pi, mi, vi, g[i], c);
    p[i] = pi;
    m[i] = mi;
    v[i] = vi;
    if (p_bf16 != nullptr) p_bf16[i] = __float2bfloat16(pi);
  }
}

// AdamW four elements per thread (16-byte fp32 accesses, 8-byte bf16 store): the same
// per-element arithmetic as adamw_kernel.
__global__ void adamw_vec_kernel(float4* __restrict__ p, const float4* __restrict__ g, float4* __restrict__ m,
                                 float4* __restrict__ v, uint2* __restrict__ p_bf16, int64_t n4, AdamWCoef c) {
  pdl_enter();
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
    float4 pi = p[i], mi = m[i], vi = v[i];
    const float4 gi = g[i];
    adamw_elem(pi.x, mi.x, vi.x, gi.x, c);
    adamw_elem(pi.y, mi.y, vi.y, gi.y, c);
    adamw_elem(pi.z, mi.z, vi.z, gi.z, c);
    adamw_elem(pi.w, mi.w, vi.w, gi.w, c);
    p[i] = pi;
    m[i] = mi;
    v[i] = vi;
    if (p_bf16 != nullptr) p_bf16[i] = make_uint2(pack_bf16(pi.x, pi.y), pack_bf16(pi.z, pi.w));
  }
}

// out[t, :] = W[id_t - start, :] if the id falls in this rank's vocab shard, else 0.
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ w,
                                     __nv_bfloat16* __restrict__ out, int rows, int d, int64_t start, int64_t count) {
  pdl_enter();
  const int t = blockIdx.x;
  if (t >= rows) return;
  const int64_t id = ids[t] - start;
  const bool mine = id >= 0 && id < count;
  uint4* dst = reinterpret_cast<uint4*>(out + int64_t(t) * d);
  const uint4* src = reinterpret_cast<const uint4*>(w + (mine ? id : 0) * d);
  for (int c = threadIdx.x; c < d / 8; c += blockDim.x) dst[c] = mine ? src[c] : make_uint4(0, 0, 0, 0);
}

// Deterministic embedding backward without a library sort. For each segment of up to
// kSortMax tokens (in token order): one CTA sorts the packed keys (local vocabulary row
// << 32 | token index) ascending in shared memory with a bitonic network -- equal rows
// keep token order, as the token index is the low word -- then one block per run of
// equal rows sums that run's dy rows in token order into dW. Tokens outside this rank's
// vocabulary shard get the largest key and are skipped. Segments are processed in
// token order, so every dW element is accumulated in the same order on every run.
constexpr int kSortMax = 16384;        // keys per segment (128 KB of shared memory)
constexpr int kSortThreads = 1024;

__global__ void __launch_bounds__(kSortThreads) embedding_sort_kernel(const int64_t* __restrict__ ids, int rows,
                                                                        int64_t start, int64_t count,
                                                                        uint64_t* __restrict__ keys_out) {
  pdl_enter();
  extern __shared__ uint64_t key[];
  int n = 1;
  while (n < rows) n <<= 1;
  for (int i = threadIdx.x; i < n; i += kSortThreads) {
    uint64_t k = ~uint64_t(0);
    if (i < rows) {
      const int64_t local = ids[i] - start;
      if (local >= 0 && local < count) k = (uint64_t(local) << 32) | uint64_t(i);
    }
    key[i] = k;
  }
  __syncthreads();
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n / 2; i += kSortThreads) {
        // the i-th compare-exchange pair of this pass
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool ascending = (lo & size) == 0;
        const uint64_t a = key[lo], b = key[hi];
        if ((a > b) == ascending) {
          key[lo] = b;
          key[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < rows; i += kSortThreads) keys_out[i] = key[i];
}

// One block per run of equal rows in the sorted keys: dW[row] += sum of the run's dy rows.
__global__ void embedding_bwd_kernel(const uint64_t* __restrict__ keys, const __nv_bfloat16* __restrict__ dy,
                                     float* __restrict__ dw, int rows, int d) {
  pdl_enter();
  const int head = blockIdx.x;
  if (head >= rows) return;
  const uint64_t k = keys[head];
  if (k == ~uint64_t(0)) return;                                 // outside this shard
  const uint32_t row = uint32_t(k >> 32);
  if (head > 0 && uint32_t(keys[head - 1] >> 32) == row) return;  // not the first of its run
  int end = head + 1;
  while (end < rows && keys[end] != ~uint64_t(0) && uint32_t(keys[end] >> 32) == row) ++end;
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float acc = 0.f;
    for (int j = head; j < end; ++j) acc += bf(dy[int64_t(uint32_t(keys[j])) * d + c]);
    dw[int64_t(row) * d + c] += acc;
  }
}

int grid_for(int64_t work, int block, int num_sms) {
  int64_t g = (work + block - 1) / block;
  return int(std::max<int64_t>(1, std::min<int64_t>(g, int64_t(num_sms) * 16)));
}

}  // namespace

void rope(void* qkv, const float* cs, int rows, int seq, int heads_qk, int hd, int64_t row_stride, int pos_offset,
          bool inverse, int num_sms, cudaStream_t st) {
  RESIHP_CHECK(hd % 2 == 0, "rope head_dim must be even");
  if (hd % 16 == 0 && row_stride % 8 == 0 && reinterpret_cast<uintptr_t>(qkv) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(cs) % 16 == 0 && pos_offset >= 0) {
    const int per_row = heads_qk * (hd / 16);
    const int block = per_row >= 256 ? 256 : ((per_row + 31) / 32) * 32;
    const int grid = std::max(1, std::min(rows, num_sms * (2048 / block)));
    launch_pdl(rope_vec_kernel, grid, block, 0, st, static_cast<__nv_bfloat16*>(qkv), reinterpret_cast<const float2*>(cs),
                                            rows, seq, heads_qk, hd, row_stride, pos_offset, inverse ? -1.f : 1.f);
    RESIHP_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const int64_t work = int64_t(rows) * heads_qk * (hd / 2);
  launch_pdl(rope_kernel, grid_for(work, 256, num_sms), 256, 0, st, static_cast<__nv_bfloat16*>(qkv),
                                                             reinterpret_cast<const float2*>(cs), rows, seq, heads_qk,
                                                             hd, row_stride, pos_offset, inverse ? -1.f : 1.f);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

void swiglu_fwd(const void* gu, void* h, int rows, int f, int num_sms, cudaStream_t st) {
  RESIHP_CHECK(f % 2 == 0, "swiglu width must be even");
  if (f % 8 == 0 && int64_t(rows) * (f / 8) < (int64_t(1) << 31) &&
      (reinterpret_cast<uintptr_t>(gu) | reinterpret_cast<uintptr_t>(h)) % 16 == 0) {
    launch_pdl(swiglu_fwd_vec_kernel, grid_for(int64_t(rows) * f / 8, 256, num_sms), 256, 0, st,
        static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(h), rows, f);
    RESIHP_CUDA_CHECK(cudaGetLastError());
    return;
  }
  launch_pdl(swiglu_fwd_kernel, grid_for(int64_t(rows) * f / 2, 256, num_sms), 256, 0, st,
      static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(h), rows, f);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

void swiglu_bwd(const void* gu, const void* dh, void* dgu, int rows, int f, int num_sms, cudaStream_t st) {
  RESIHP_CHECK(f % 2 == 0, "swiglu width must be even");
  if (f % 8 == 0 && int64_t(rows) * (f / 8) < (int64_t(1) << 31) &&
      (reinterpret_cast<uintptr_t>(gu) | reinterpret_cast<uintptr_t>(dh) | reinterpret_cast<uintptr_t>(dgu)) % 16 == 0) {
    launch_pdl(swiglu_bwd_vec_kernel, grid_for(int64_t(rows) * f / 8, 256, num_sms), 256, 0, st,
        static_cast<const __nv_bfloat16*>(gu), static_cast<const __nv_bfloat16*>(dh), static_cast<__nv_bfloat16*>(dgu),
        rows, f);
    RESIHP_CUDA_CHECK(cudaGetLastError());
    return;
  }
  launch_pdl(swiglu_bwd_kernel, grid_for(int64_t(rows) * f / 2, 256, num_sms), 256, 0, st,
      static_cast<const __nv_bfloat16*>(gu), static_cast<const __nv_bfloat16*>(dh), static_cast<__nv_bfloat16*>(dgu),
      rows, f);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

AdamWCoef adamw_coef(float lr, float b1, float b2, float eps, float wd, int64_t step, float grad_scale) {
  RESIHP_CHECK(step >= 1, "AdamW step must be >= 1");
  const double bc1 = 1.0 - std::pow(double(b1), double(step));
  const double bc2 = 1.0 - std::pow(double(b2), double(step));
  AdamWCoef c;
  c.lr = lr;
  c.b1 = b1;
  c.b2 = b2;
  c.eps = eps;
  c.wd = wd;
  c.step_size = float(double(lr) / bc1);
  c.bc2_sqrt = float(std::sqrt(bc2));
  c.grad_scale = grad_scale;
  return c;
}

void adamw(float* p, const float* g, float* m, float* v, void* p_bf16, int64_t n, float lr, float b1, float b2,
           float eps, float wd, int64_t step, float grad_scale, int num_sms, cudaStream_t st) {
  const AdamWCoef c = adamw_coef(lr, b1, b2, eps, wd, step, grad_scale);
  const uintptr_t al = reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) |
                       reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v);
  if (n % 4 == 0 && al % 16 == 0 && reinterpret_cast<uintptr_t>(p_bf16) % 8 == 0) {
    launch_pdl(adamw_vec_kernel, grid_for(n / 4, 256, num_sms), 256, 0, st,
        reinterpret_cast<float4*>(p), reinterpret_cast<const float4*>(g), reinterpret_cast<float4*>(m),
        reinterpret_cast<float4*>(v), static_cast<uint2*>(p_bf16), n / 4, c);
    RESIHP_CUDA_CHECK(cudaGetLastError());
    return;
  }
  launch_pdl(adamw_kernel, grid_for(n, 256, num_sms), 256, 0, st, p, g, m, v, static_cast<__nv_bfloat16*>(p_bf16), n, c);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

void embedding_fwd(const int64_t* ids, const void* w, void* out, int rows, int d, int64_t start, int64_t count,
                   cudaStream_t st) {
  RESIHP_CHECK(d % 8 == 0, "embedding width must be a multiple of 8");
  launch_pdl(embedding_fwd_kernel, rows, 128, 0, st, ids, static_cast<const __nv_bfloat16*>(w),
                                             static_cast<__nv_bfloat16*>(out), rows, d, start, count);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

int embedding_sort_segment() { return kSortMax; }

void embedding_bwd(const int64_t* ids, const void* dy, float* dw, uint64_t* keys, int rows, int d, int64_t start,
                   int64_t count, cudaStream_t st) {
  RESIHP_CHECK(count < (int64_t(1) << 32) - 1, "embedding shard too large for 32-bit row keys");
  const auto* dyb = static_cast<const __nv_bfloat16*>(dy);
  const int smem = kSortMax * int(sizeof(uint64_t));
  RESIHP_CUDA_CHECK(cudaFuncSetAttribute(embedding_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  for (int off = 0; off < rows; off += kSortMax) {
    const int seg = std::min(kSortMax, rows - off);
    int n = 1;
    while (n < seg) n <<= 1;
    launch_pdl(embedding_sort_kernel, 1, kSortThreads, n * int(sizeof(uint64_t)), st, ids + off, seg, start, count, keys);
    RESIHP_CUDA_CHECK(cudaGetLastError());
    launch_pdl(embedding_bwd_kernel, seg, 256, 0, st, keys, dyb + int64_t(off) * d, dw, seg, d);
    RESIHP_CUDA_CHECK(cudaGetLastError());
  }
}

}  // namespace resihp
