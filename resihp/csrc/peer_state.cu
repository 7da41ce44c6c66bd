// Peer-memory kernels over a stage's flat training state. Each rank keeps its FP32
// master weights, Adam moments and two gradient buffers in one CUDA-IPC-exported region;
// the ranks that share work map each other's regions and read them with plain P2P loads
// over NVLink (nothing here is multicast, no library kernel touches a peer pointer).
//
// * dp_allreduce_adamw -- the data-parallel gradient all-reduce fused with the AdamW
//   step and the bf16 refresh of the compute weights (reference: the CPU object gather
//   of resihp/parallel/dp.py:98-151 followed by the optimizer step at
//   resihp/parallel/pp.py:428-451). Every DP rank reads its peers' accumulated gradients
//   straight from their regions, sums them in ascending group-rank order (the same bits
//   on every replica, independent of arrival order), applies AdamW to its own copy of the
//   replicated state and writes the sum into its second gradient buffer, which becomes
//   the visible gradient for the step. One launch replaces all-reduce + AdamW.
// * reshard_gather -- the post-failure state move (reference: resihp/parallel/reshard.py
//   :187-243 and resihp/recovery.py:373-468): the new owner of a shard pulls every piece
//   of it from the donors' regions with the re-partition (new TP degree, shard dim 0 or 1)
//   folded into the copy descriptors, and writes the bf16 compute copy of the master
//   weights in the same pass.
#include <atomic>
#include <cuda_bf16.h>

#include "common.cuh"
#include "launch.h"

namespace resihp {

namespace {
std::atomic<uint64_t> g_peer_wait_budget_ns{kWaitBudgetNs};
}  // namespace

uint64_t peer_wait_budget_ns() { return g_peer_wait_budget_ns.load(std::memory_order_relaxed); }

void set_peer_wait_budget_ns(uint64_t ns) {
  RESIHP_CHECK(ns > 0, "peer wait budget must be positive");
  g_peer_wait_budget_ns.store(ns, std::memory_order_relaxed);
}

// ---- fused DP all-reduce + AdamW -----------------------------------------------------

constexpr int kDpThreads = 512;

// Float4 groups per thread per iteration: as many as the registers allow at a bound of
// 128 per thread (one 512-thread CTA per SM), so enough peer loads are in flight to
// cover the NVLink round trip.
template <int Q>
__host__ __device__ constexpr int dp_unroll() { return Q <= 2 ? 4 : (Q <= 4 ? 2 : 1); }

struct DpArgs {
  const float4* grad[kMaxDp];  // group rank q's accumulation buffer; grad[me] is local
  float4* sum_out;             // local: receives the reduced gradient
  float4* p;
  float4* m;
  float4* v;
  uint2* p_bf16;               // four bf16 per float4 (nullptr: no compute copy)
  unsigned* flags_local;       // [grid][kMaxDp], written by the peers
  unsigned* flags_peer[kMaxDp];
  int dp, me;
  unsigned epoch;
  int64_t n4, per_cta;
  AdamWCoef c;
  int* err;
  uint64_t wait_ns;            // budget of each wait on a peer's flag
  // two-phase variant only (reduce-scatter, push, local AdamW):
  float4* sum_peer[kMaxDp];    // group rank q's receiving buffer (its sum_out); [me] is local
  unsigned* flags2_local;      // [grid][kMaxDp]: "my part's sums are in your buffer", written by peers
  unsigned* flags2_peer[kMaxDp];
};

__device__ __forceinline__ float4 ld_cg_f4(const float4* p) { return __ldcg(p); }

__device__ __forceinline__ void add4(float4& a, const float4& b) {
  a.x += b.x;
  a.y += b.y;
  a.z += b.z;
  a.w += b.w;
}

__device__ __forceinline__ uint2 pack4_bf16(const float4& x) {
  return make_uint2(pack_bf16(x.x, x.y), pack_bf16(x.z, x.w));
}

// CTA b of every DP rank owns the same slice [b * per_cta, (b + 1) * per_cta) of the flat
// buffers, so the cross-GPU handshake is per CTA pair: b announces "my gradients for this
// epoch are final" in each peer's flag array, then waits for every peer's announcement.
// The gradients were written by earlier kernels on this stream (complete before this
// launch), so the release store publishes them; the peer's acquire load plus the CTA
// barrier orders every later read of them. A peer that has already moved on to the next
// epoch can only do so after this rank's announcement, and it then writes only its own
// second buffer, never the one read here -- hence ">=".
template <int Q>  // compile-time bound on the group size (2, 4 or 8): keeps the loads in registers
__global__ void __launch_bounds__(kDpThreads) dp_adamw_kernel(const __grid_constant__ DpArgs a) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    int good = 1;
    __threadfence_system();
    for (int q = 0; q < a.dp; ++q)
      if (q != a.me) st_release_sys(a.flags_peer[q] + blockIdx.x * kMaxDp + a.me, a.epoch);
    for (int q = 0; q < a.dp && good; ++q)
      if (q != a.me && !wait_geq(a.flags_local + blockIdx.x * kMaxDp + q, a.epoch, a.err, kErrPeerWait, a.wait_ns)) good = 0;
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  const int64_t lo = int64_t(blockIdx.x) * a.per_cta;
  const int64_t hi = lo + a.per_cta < a.n4 ? lo + a.per_cta : a.n4;
  constexpr int kDpUnroll = dp_unroll<Q>();
  constexpr int64_t kStep = int64_t(kDpThreads) * kDpUnroll;
  for (int64_t base = lo + threadIdx.x; base < hi; base += kStep) {
    float4 g[Q][kDpUnroll];
    float4 p[kDpUnroll], m[kDpUnroll], v[kDpUnroll];
    // Issue every load of this iteration before using any of them (the peer reads cross
    // NVLink; their latency is hidden behind each other and behind the local streams).
    #pragma unroll
    for (int u = 0; u < kDpUnroll; ++u) {
      const int64_t i = base + u * kDpThreads;
      if (i >= hi) continue;
      #pragma unroll
      for (int q = 0; q < Q; ++q)
        if (q < a.dp) g[q][u] = ld_cg_f4(a.grad[q] + i);
      p[u] = __ldcs(a.p + i);
      m[u] = __ldcs(a.m + i);
      v[u] = __ldcs(a.v + i);
    }
    #pragma unroll
    for (int u = 0; u < kDpUnroll; ++u) {
      const int64_t i = base + u * kDpThreads;
      if (i >= hi) continue;
      float4 s = g[0][u];
      #pragma unroll
      for (int q = 1; q < Q; ++q)
        if (q < a.dp) add4(s, g[q][u]);
      a.sum_out[i] = s;
      adamw_elem(p[u].x, m[u].x, v[u].x, s.x, a.c);
      adamw_elem(p[u].y, m[u].y, v[u].y, s.y, a.c);
      adamw_elem(p[u].z, m[u].z, v[u].z, s.z, a.c);
      adamw_elem(p[u].w, m[u].w, v[u].w, s.w, a.c);
      __stcs(a.p + i, p[u]);
      __stcs(a.m + i, m[u]);
      __stcs(a.v + i, v[u]);
      if (a.p_bf16 != nullptr) a.p_bf16[i] = pack4_bf16(p[u]);
    }
  }
}

// Two-phase variant for larger groups: CTA b of every rank still owns the same slice of
// the flat buffers, but the slice is cut into `dp` parts and group rank q reduces only
// part q. Phase 1: rank q sums part q of every rank's accumulated gradient (rank order,
// so the bits are the same as the one-phase kernel's) and *pushes* the sum into part q
// of every rank's receiving buffer (its own with a local store). Phase 2: once every
// peer has flagged its part as pushed, each rank applies AdamW to the whole slice from
// its now complete local receiving buffer. NVLink carries 2 (dp-1)/dp of the gradient
// bytes into each GPU instead of (dp-1) times them.
//
// Buffer safety: the pushes of step t land in each rank's receiving buffer for step t,
// which nobody reads or writes in step t before the pushes (its owner accumulates into
// the other buffer, and the previous step's readers of it -- phase 1 of step t-1 --
// finished before their step-t announcement, which the pusher waited for in phase 0).
// A rank leaves the kernel only after every push into it is flagged, so its next step
// can zero and reuse the buffer freely.
template <int Q>
__global__ void __launch_bounds__(kDpThreads) dp_adamw_push_kernel(const __grid_constant__ DpArgs a) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    int good = 1;
    __threadfence_system();
    for (int q = 0; q < a.dp; ++q)
      if (q != a.me) st_release_sys(a.flags_peer[q] + blockIdx.x * kMaxDp + a.me, a.epoch);
    for (int q = 0; q < a.dp && good; ++q)
      if (q != a.me && !wait_geq(a.flags_local + blockIdx.x * kMaxDp + q, a.epoch, a.err, kErrPeerWait, a.wait_ns))
        good = 0;
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  const int64_t lo = int64_t(blockIdx.x) * a.per_cta;
  const int64_t hi = lo + a.per_cta < a.n4 ? lo + a.per_cta : a.n4;
  const int64_t part = (hi - lo + a.dp - 1) / a.dp;
  const int64_t mlo = lo + a.me * part < hi ? lo + a.me * part : hi;
  const int64_t mhi = mlo + part < hi ? mlo + part : hi;
  constexpr int kU = dp_unroll<Q>();
  constexpr int64_t kStep = int64_t(kDpThreads) * kU;
  // phase 1: reduce my part, push it to every rank
  for (int64_t base = mlo + threadIdx.x; base < mhi; base += kStep) {
    float4 g[Q][kU];
    #pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * kDpThreads;
      if (i >= mhi) continue;
      #pragma unroll
      for (int q = 0; q < Q; ++q)
        if (q < a.dp) g[q][u] = ld_cg_f4(a.grad[q] + i);
    }
    #pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * kDpThreads;
      if (i >= mhi) continue;
      float4 s = g[0][u];
      #pragma unroll
      for (int q = 1; q < Q; ++q)
        if (q < a.dp) add4(s, g[q][u]);
      #pragma unroll
      for (int q = 0; q < Q; ++q)
        if (q < a.dp) __stcg(a.sum_peer[q] + i, s);
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    int good = 1;
    for (int q = 0; q < a.dp; ++q)
      if (q != a.me) st_release_sys(a.flags2_peer[q] + blockIdx.x * kMaxDp + a.me, a.epoch);
    for (int q = 0; q < a.dp && good; ++q)
      if (q != a.me && !wait_geq(a.flags2_local + blockIdx.x * kMaxDp + q, a.epoch, a.err, kErrPeerWait, a.wait_ns))
        good = 0;
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  // phase 2: AdamW over the whole slice from the local receiving buffer
  for (int64_t base = lo + threadIdx.x; base < hi; base += kStep) {
    float4 s[kU], p[kU], m[kU], v[kU];
    #pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * kDpThreads;
      if (i >= hi) continue;
      s[u] = __ldcg(a.sum_out + i);
      p[u] = __ldcs(a.p + i);
      m[u] = __ldcs(a.m + i);
      v[u] = __ldcs(a.v + i);
    }
    #pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * kDpThreads;
      if (i >= hi) continue;
      adamw_elem(p[u].x, m[u].x, v[u].x, s[u].x, a.c);
      adamw_elem(p[u].y, m[u].y, v[u].y, s[u].y, a.c);
      adamw_elem(p[u].z, m[u].z, v[u].z, s[u].z, a.c);
      adamw_elem(p[u].w, m[u].w, v[u].w, s[u].w, a.c);
      __stcs(a.p + i, p[u]);
      __stcs(a.m + i, m[u]);
      __stcs(a.v + i, v[u]);
      if (a.p_bf16 != nullptr) a.p_bf16[i] = pack4_bf16(p[u]);
    }
  }
}

int dp_grid(int64_t n, int num_sms) {
  const int64_t n4 = n / 4;
  const int64_t want = 2 * int64_t(num_sms);
  const int64_t per = (n4 + want - 1) / want;
  return int(per > 0 ? (n4 + per - 1) / per : 1);
}

void dp_allreduce_adamw(const float* const* grads, int dp, int me, float* sum_out, float* p, float* m, float* v,
                        void* p_bf16, int64_t n, const AdamWCoef& coef, unsigned* flags_local,
                        unsigned* const* flags_peer, unsigned epoch, int grid, int* err, cudaStream_t st,
                        float* const* sums_peer, unsigned* flags2_local, unsigned* const* flags2_peer) {
  RESIHP_CHECK(dp >= 1 && dp <= kMaxDp && me >= 0 && me < dp, "dp_allreduce_adamw: bad group size / rank");
  RESIHP_CHECK(n % 4 == 0 && n > 0, "dp_allreduce_adamw: buffer length must be a positive multiple of 4");
  RESIHP_CHECK(grid >= 1, "dp_allreduce_adamw: empty grid");
  DpArgs a{};
  for (int q = 0; q < dp; ++q) {
    RESIHP_CHECK(reinterpret_cast<uintptr_t>(grads[q]) % 16 == 0, "dp_allreduce_adamw: unaligned gradient buffer");
    a.grad[q] = reinterpret_cast<const float4*>(grads[q]);
    a.flags_peer[q] = flags_peer[q];
  }
  a.sum_out = reinterpret_cast<float4*>(sum_out);
  a.p = reinterpret_cast<float4*>(p);
  a.m = reinterpret_cast<float4*>(m);
  a.v = reinterpret_cast<float4*>(v);
  a.p_bf16 = static_cast<uint2*>(p_bf16);
  a.flags_local = flags_local;
  a.dp = dp;
  a.me = me;
  a.epoch = epoch;
  a.n4 = n / 4;
  a.per_cta = (a.n4 + grid - 1) / grid;
  a.c = coef;
  a.err = err;
  a.wait_ns = peer_wait_budget_ns();
  if (sums_peer != nullptr) {
    RESIHP_CHECK(flags2_local != nullptr && flags2_peer != nullptr, "dp_allreduce_adamw: push variant needs flags");
    for (int q = 0; q < dp; ++q) {
      RESIHP_CHECK(reinterpret_cast<uintptr_t>(sums_peer[q]) % 16 == 0, "dp_allreduce_adamw: unaligned sum buffer");
      a.sum_peer[q] = reinterpret_cast<float4*>(sums_peer[q]);
      a.flags2_peer[q] = flags2_peer[q];
    }
    RESIHP_CHECK(a.sum_peer[me] == a.sum_out, "dp_allreduce_adamw: sums_peer[me] must be the local sum buffer");
    a.flags2_local = flags2_local;
    if (dp <= 2) dp_adamw_push_kernel<2><<<grid, kDpThreads, 0, st>>>(a);
    else if (dp <= 4) dp_adamw_push_kernel<4><<<grid, kDpThreads, 0, st>>>(a);
    else dp_adamw_push_kernel<8><<<grid, kDpThreads, 0, st>>>(a);
  } else if (dp <= 2) {
    dp_adamw_kernel<2><<<grid, kDpThreads, 0, st>>>(a);
  } else if (dp <= 4) {
    dp_adamw_kernel<4><<<grid, kDpThreads, 0, st>>>(a);
  } else {
    dp_adamw_kernel<8><<<grid, kDpThreads, 0, st>>>(a);
  }
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

// ---- reshard gather --------------------------------------------------------------------

constexpr int kCopyThreads = 256;

// Work item -> descriptor (descriptors are sorted by item_base).
__device__ __forceinline__ int find_desc(const CopyDesc* d, int nd, int64_t item) {
  int lo = 0, hi = nd - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (d[mid].item_base <= item) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// One CTA copies one row of one descriptor per iteration (rows are at most a few tens of
// thousands of elements: the host splits long contiguous runs).
__global__ void __launch_bounds__(kCopyThreads) reshard_gather_kernel(const CopyDesc* __restrict__ descs, int nd,
                                                                      int64_t items, int* err) {
  __shared__ CopyDesc sd;
  for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
    __syncthreads();
    if (threadIdx.x == 0) sd = descs[find_desc(descs, nd, item)];
    __syncthreads();
    const int64_t r = item - sd.item_base;
    if (r < 0 || r >= sd.rows) {
      if (threadIdx.x == 0) record_error(err, kErrBounds);
      continue;
    }
    const float* src = sd.src + r * sd.src_ld;
    float* dst = sd.dst + r * sd.dst_ld;
    __nv_bfloat16* dst16 = sd.dst_bf16 == nullptr ? nullptr : static_cast<__nv_bfloat16*>(sd.dst_bf16) + r * sd.dst_ld;
    if (sd.vec4) {
      const int64_t c4 = sd.cols / 4;
      const float4* s4 = reinterpret_cast<const float4*>(src);
      float4* d4 = reinterpret_cast<float4*>(dst);
      constexpr int kU = 4;
      for (int64_t c = threadIdx.x; c < c4; c += int64_t(kCopyThreads) * kU) {
        float4 x[kU];
        #pragma unroll
        for (int u = 0; u < kU; ++u)
          if (c + u * kCopyThreads < c4) x[u] = __ldcg(s4 + c + u * kCopyThreads);
        #pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int64_t j = c + u * kCopyThreads;
          if (j >= c4) continue;
          d4[j] = x[u];
          if (dst16 != nullptr) reinterpret_cast<uint2*>(dst16)[j] = pack4_bf16(x[u]);
        }
      }
    } else {
      for (int64_t c = threadIdx.x; c < sd.cols; c += kCopyThreads) {
        const float x = __ldcg(src + c);
        dst[c] = x;
        if (dst16 != nullptr) dst16[c] = __float2bfloat16(x);
      }
    }
  }
}

void reshard_gather(const CopyDesc* descs_device, int ndesc, int64_t items, int* err, int num_sms, cudaStream_t st) {
  if (ndesc == 0 || items == 0) return;
  const int64_t cap = int64_t(num_sms) * 8;
  const int grid = int(items < cap ? items : cap);
  reshard_gather_kernel<<<grid, kCopyThreads, 0, st>>>(descs_device, ndesc, items, err);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

}  // namespace resihp
