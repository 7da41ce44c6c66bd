// Tensor-parallel GEMMs fused with their sequence-parallel collective over NVLink peer
// memory (CUDA IPC mappings of each rank's symmetric workspace; plain P2P loads,
// stores and atomics -- no multicast of any kind).
//
//   AG->GEMM   y[T, N]  = all_gather_tokens(x_r[T/tp, K]) * W[N, K]^T
//   GEMM->RS   y_r[T/tp, N] = reduce_scatter_tokens(h[T, K] * W[N, K]^T)
//
// Both are the persistent tcgen05 GEMM of gemm.cu (TMA producer warp, one MMA-issuing
// thread, four epilogue warps, two TMEM accumulators) with the collective woven in:
//
// AG: tiles run chunk by chunk, this rank's own token chunk first (read in place through
// its own tensor map). Two extra copy warps per CTA pull this CTA's share of every peer's
// chunk over NVLink -- each remote byte crosses the link once -- into the local gather
// buffer, then bump that chunk's ready counter; the producer waits for a chunk's counter
// before its first TMA load from the gather buffer. The gather buffer ends up holding
// the whole gathered input, which the backward pass reuses for the weight gradient.
// A rank's chunk is published (copied into its symmetric slot, then flagged to every
// peer) by ag_publish_kernel; slots alternate by epoch parity, and a rank only
// overwrites a slot once every peer has published the next epoch, i.e. has finished
// reading the previous one.
//
// RS: tiles of the peers' token chunks run first; their epilogue stores the bf16
// partial tile straight into the owner's receive slot (this rank's row of it) and bumps
// the owner's arrival counter for this source. The own chunk runs last: its epilogue
// waits for every source's tiles, then sums the partials in rank order (fp32) and writes
// the reduced rows -- deterministic, and the reduction costs no extra pass.
//
// Every wait (peer flags, counters, mbarriers) is bounded by the global timer and
// reports into the error word. Both kernels rely on all their CTAs being resident at once
// (grid <= SM count, one CTA per SM); if that ever fails, the bounded waits turn it into
// an error instead of a hang.
#include <algorithm>
#include <cstring>
#include <cooperative_groups.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "launch.h"

namespace resihp {

constexpr int kMaxTp = 8;

struct CommArgs {
  int rank, tp, rows_per_rank;
  unsigned epoch;
  // AG
  const __nv_bfloat16* peer_x[kMaxTp];  // each rank's published slot for this call
  __nv_bfloat16* xg;                     // local gather buffer [T, K]
  const __nv_bfloat16* x_local;          // this rank's chunk [T/tp, K]
  int64_t ldx;
  unsigned* sig_ag;                      // local: sig_ag[s] = last epoch rank s published
  unsigned* ready;                       // local per-chunk ready counters [tp]
  unsigned ready_target;
  // RS
  __nv_bfloat16* peer_recv[kMaxTp];      // each rank's receive slot base for this call
  unsigned* peer_arrive[kMaxTp];         // each rank's arrival counters [tp]
  unsigned* peer_sig_rs[kMaxTp];         // each rank's sig_rs array [tp]
  unsigned* arrive;                      // local arrival counters [tp]
  unsigned* sig_rs;                      // local sig_rs array [tp]
  unsigned arrive_target;
  __nv_bfloat16* recv_local;             // local receive slot base for this call
};

struct FusedArgs {
  void* c;          // AG: y [T, N]; RS: y_r [T/tp, N]
  int64_t ldc;
  int m, n, k;
  int* err;
  CommArgs comm;
};

// ---- memory-model helpers ------------------------------------------------------------

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Wait until *p >= target (wrap-safe); false + error code when the budget runs out.
__device__ __forceinline__ bool wait_geq(const unsigned* p, unsigned target, int* err, int code) {
  const uint64_t start = globaltimer();
  #pragma unroll 1
  while (static_cast<int>(ld_acquire_sys(p) - target) < 0) {
    if (globaltimer() - start > kWaitBudgetNs) {
      record_error(err, code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// ---- tile order ------------------------------------------------------------------------

constexpr int kFBM = 128;
constexpr int kFBK = 64;

template <int BN>
struct FusedShape {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = kFBM * kFBK * 2;
  static constexpr int kBBytes = BN * kFBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
};

// Tile t -> (chunk, m0, n0). Chunks are visited starting at (rank + first) % tp; inside a
// chunk, tiles are grouped along M for L2 reuse.
__device__ __forceinline__ void fused_tile(int t, int tiles_m_chunk, int tiles_n, const CommArgs& c, int first,
                                           int& chunk, int& m0, int& tn_out) {
  const int per_chunk = tiles_m_chunk * tiles_n;
  const int pos = t / per_chunk;
  const int local = t % per_chunk;
  chunk = (c.rank + first + pos) % c.tp;
  constexpr int kGroup = 8;
  const int per_group = kGroup * tiles_n;
  const int group = local / per_group;
  const int g0 = group * kGroup;
  const int size = min(tiles_m_chunk - g0, kGroup);
  const int in_group = local % per_group;
  const int tm = g0 + in_group % size;
  const int tn = in_group / size;
  m0 = chunk * c.rows_per_rank + tm * kFBM;
  tn_out = tn;
}

template <int BN, bool B_MN, int MODE>
__global__ void __launch_bounds__(MODE == 1 ? 256 : 192, 1)
    fused_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_a2,
                      const __grid_constant__ CUtensorMap tma_b, FusedArgs g) {
  using S = FusedShape<BN>;
  constexpr int kStages = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * S::kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const CommArgs& cm = g.comm;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m_chunk = cm.rows_per_rank / kFBM;
  const int tiles_n = (g.n + BN - 1) / BN;
  const int tiles = tiles_m_chunk * tiles_n * cm.tp;
  const int kblocks = (g.k + kFBK - 1) / kFBK;
  const int first = MODE == 1 ? 0 : 1;  // AG: own chunk first; RS: own chunk last

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    fence_barrier_init();
    if (MODE == 2 && blockIdx.x == 0) {
      // "I started RS epoch e": every slot of epoch e-1 has been read here.
      for (int p = 0; p < cm.tp; ++p)
        if (p != cm.rank) st_release_sys(cm.peer_sig_rs[p] + cm.rank, cm.epoch);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch(&tma_a);
      tma_prefetch(&tma_b);
      if (MODE == 1) tma_prefetch(&tma_a2);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int ready_chunk = -1;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int chunk, m0, tn;
        fused_tile(t, tiles_m_chunk, tiles_n, cm, first, chunk, m0, tn);
        const int n0 = tn * BN;
        const bool own = chunk == cm.rank;
        if (MODE == 1 && !own && ready_chunk != chunk) {
          if (!wait_geq(cm.ready + chunk, cm.ready_target, g.err, kErrPeerWait)) { ok = false; break; }
          fence_proxy_async_global();
          ready_chunk = chunk;
        }
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, g.err, kErrTmaWait)) { ok = false; break; }
          uint8_t* sa = smem + s * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_expect_tx(&full[s], S::kStageBytes);
          const int k0 = kb * kFBK;
          if (MODE == 1 && own) tma_load_2d(sa, &tma_a, &full[s], k0, m0 - cm.rank * cm.rows_per_rank);
          else if (MODE == 1) tma_load_2d(sa, &tma_a2, &full[s], k0, m0);
          else tma_load_2d(sa, &tma_a, &full[s], k0, m0);
          if (B_MN) {
            #pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_2d(sb + c * 8192, &tma_b, &full[s], n0 + 64 * c, k0);
          } else {
            tma_load_2d(sb, &tma_b, &full[s], k0, n0);
          }
          if (++s == kStages) { s = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kFBM, BN, 0, B_MN ? 1 : 0);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int i = 0;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
        const int a = i & 1;
        const uint32_t accph = (i >> 1) & 1;
        if (!mbar_wait(&acc_empty[a], accph ^ 1, g.err, kErrMmaWait)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + a * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[s], ph, g.err, kErrMmaWait)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * S::kStageBytes);
          const uint32_t sb = sa + S::kABytes;
          #pragma unroll
          for (int kk = 0; kk < kFBK / 16; ++kk) {
            const uint64_t da = smem_desc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t db = B_MN ? smem_desc_sw128(sb + kk * 2048, 8192, 1024) : smem_desc_sw128(sb + kk * 32, 16, 1024);
            umma_bf16(d, da, db, idesc, (kb | kk) != 0);
          }
          umma_commit(&empty[s]);
          if (++s == kStages) { s = 0; ph ^= 1; }
        }
        umma_commit(&acc_full[a]);
      }
    }
  } else if (warp < 6) {
    const int q = warp & 3;
    int i = 0;
    bool remote_ok[kMaxTp];
    #pragma unroll
    for (int p = 0; p < kMaxTp; ++p) remote_ok[p] = false;
    bool own_ready = false;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
      int chunk, m0, tn;
      fused_tile(t, tiles_m_chunk, tiles_n, cm, first, chunk, m0, tn);
      const int a = i & 1;
      const uint32_t accph = (i >> 1) & 1;
      if (!mbar_wait(&acc_full[a], accph, g.err, kErrEpiWait)) break;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;             // global row in [0, T)
      const int lrow = row - chunk * cm.rows_per_rank;  // row inside its chunk
      __nv_bfloat16* dst;
      int64_t ld;
      if (MODE == 1) {
        dst = static_cast<__nv_bfloat16*>(g.c) + int64_t(row) * g.ldc;
        ld = g.ldc;
      } else if (chunk != cm.rank) {
        // wait once per owner: its slot of this parity is free again
        if (!remote_ok[chunk]) {
          if (cm.epoch > 1 && lane == 0 &&
              !wait_geq(cm.sig_rs + chunk, cm.epoch - 1, g.err, kErrPeerWait))
            ok = false;
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
          remote_ok[chunk] = true;
        }
        dst = cm.peer_recv[chunk] + (int64_t(cm.rank) * cm.rows_per_rank + lrow) * g.n;
        ld = g.n;
      } else {
        if (!own_ready) {
          if (lane == 0) {
            for (int p = 0; p < cm.tp && ok; ++p)
              if (p != cm.rank && !wait_geq(cm.arrive + p, cm.arrive_target, g.err, kErrPeerWait)) ok = false;
          }
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
          own_ready = true;
        }
        dst = static_cast<__nv_bfloat16*>(g.c) + int64_t(lrow) * g.ldc;
        ld = g.ldc;
      }
      (void)ld;
      #pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t v[32];
        tmem_ld32(tmem_base + a * BN + cc * 32 + (uint32_t(q * 32) << 16), v);
        tmem_wait_ld();
        const int col0 = tn * BN + cc * 32;
        if (!ok || col0 >= g.n) continue;
        float f[32];
        #pragma unroll
        for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(v[e]);
        if (MODE == 2 && chunk == cm.rank) {
          // rank-ordered sum of every source's partial (own partial in fp32)
          float tot[32];
          #pragma unroll
          for (int e = 0; e < 32; ++e) tot[e] = 0.f;
          for (int src = 0; src < cm.tp; ++src) {
            if (src == cm.rank) {
              #pragma unroll
              for (int e = 0; e < 32; ++e) tot[e] += f[e];
            } else {
              const __nv_bfloat16* p = cm.recv_local + (int64_t(src) * cm.rows_per_rank + lrow) * g.n + col0;
              #pragma unroll
              for (int u = 0; u < 4; ++u) {
                uint4 raw4 = *reinterpret_cast<const uint4*>(p + 8 * u);
                const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw4);
                #pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 x = __bfloat1622float2(h[e]);
                  tot[8 * u + 2 * e] += x.x;
                  tot[8 * u + 2 * e + 1] += x.y;
                }
              }
            }
          }
          #pragma unroll
          for (int e = 0; e < 32; ++e) f[e] = tot[e];
        }
        #pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 o;
          o.x = pack_bf16(f[8 * u + 0], f[8 * u + 1]);
          o.y = pack_bf16(f[8 * u + 2], f[8 * u + 3]);
          o.z = pack_bf16(f[8 * u + 4], f[8 * u + 5]);
          o.w = pack_bf16(f[8 * u + 6], f[8 * u + 7]);
          *reinterpret_cast<uint4*>(dst + col0 + 8 * u) = o;
        }
      }
      if (MODE == 2 && chunk != cm.rank) {
        // publish this warp's 32 rows of the tile: fence the stores system-wide, then
        // one lane bumps the owner's counter (four arrivals per tile, one per warp)
        __threadfence_system();
        __syncwarp();
        if (lane == 0) atomicAdd_system(cm.peer_arrive[chunk] + cm.rank, 1u);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
  } else if (MODE == 1) {
    // copy warps: this CTA's share of every peer chunk, then of the own chunk
    const int ct = threadIdx.x - 192;  // 0..63
    const int64_t vec_per_row = cm.ldx / 8;
    const int lo = int(int64_t(cm.rows_per_rank) * blockIdx.x / gridDim.x);
    const int hi = int(int64_t(cm.rows_per_rank) * (blockIdx.x + 1) / gridDim.x);
    bool ok = true;
    for (int p = 1; p <= cm.tp && ok; ++p) {
      const int chunk = (cm.rank + p) % cm.tp;
      const bool own = chunk == cm.rank;
      if (!own) {
        if (lane == 0 && !wait_geq(cm.sig_ag + chunk, cm.epoch, g.err, kErrPeerWait)) ok = false;
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
      const uint4* src = reinterpret_cast<const uint4*>((own ? cm.x_local : cm.peer_x[chunk]) + int64_t(lo) * cm.ldx);
      uint4* dst = reinterpret_cast<uint4*>(cm.xg + (int64_t(chunk) * cm.rows_per_rank + lo) * cm.ldx);
      const int64_t nvec = int64_t(hi - lo) * vec_per_row;
      constexpr int kUnroll = 8;
      for (int64_t base = ct; base < nvec; base += 64 * kUnroll) {
        uint4 r[kUnroll];
        #pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (base + u * 64 < nvec) r[u] = ld_cg_v4(src + base + u * 64);
        #pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (base + u * 64 < nvec) dst[base + u * 64] = r[u];
      }
      // make this warp's stores visible to the TMA (async proxy) readers, then arrive
      // (two arrivals per CTA per chunk, one per copy warp)
      fence_proxy_async_global();
      __threadfence();
      __syncwarp();
      if (lane == 0 && !own) atomicAdd(cm.ready + chunk, 1u);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// Publish this rank's chunk for AG epoch `epoch`: wait until every peer has published
// epoch-1 (so it finished reading this parity's slot at epoch-2), copy the chunk into the
// slot, and -- from the last block to finish -- flag the epoch to every peer.
struct PublishArgs {
  const uint4* x;
  uint4* slot;
  int64_t nvec;
  int rank, tp;
  unsigned epoch;
  unsigned* sig_ag;                 // local
  unsigned* peer_sig_ag[kMaxTp];    // each rank's sig_ag array
  unsigned* done;                   // local block-completion counter
  unsigned done_target;
  int* err;
};

__global__ void ag_publish_kernel(PublishArgs a) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    if (a.epoch > 1)
      for (int p = 0; p < a.tp; ++p)
        if (p != a.rank && !wait_geq(a.sig_ag + p, a.epoch - 1, a.err, kErrPeerWait)) ok = 0;
  }
  __syncthreads();
  if (!ok) return;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < a.nvec; i += int64_t(gridDim.x) * blockDim.x)
    a.slot[i] = a.x[i];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(a.done, 1u);
    if (prev + 1 == a.done_target) {
      __threadfence_system();
      for (int p = 0; p < a.tp; ++p)
        if (p != a.rank) st_release_sys(a.peer_sig_ag[p] + a.rank, a.epoch);
    }
  }
}

// ---------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------

namespace {

int sm_count() {
  int dev = 0, n = 0;
  RESIHP_CUDA_CHECK(cudaGetDevice(&dev));
  RESIHP_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  return n;
}

template <int BN, bool B_MN, int MODE>
void launch_fused(const CUtensorMap& ta, const CUtensorMap& ta2, const CUtensorMap& tb, FusedArgs g, int grid,
                  cudaStream_t st) {
  using S = FusedShape<BN>;
  auto kernel = fused_gemm_kernel<BN, B_MN, MODE>;
  RESIHP_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem));
  // The grid never exceeds the SM count and one CTA fills an SM, so on a GPU this process
  // owns every CTA is resident at once.
  kernel<<<grid, MODE == 1 ? 256 : 192, S::kSmem, st>>>(ta, ta2, tb, g);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

}  // namespace

int fused_grid(int m, int n, int tp) {
  const int tiles = (m / kFBM) * ((n + 255) / 256);
  (void)tp;
  return std::min(tiles, sm_count());
}

void ag_publish(const void* x, void* slot, int64_t bytes, int rank, int tp, unsigned epoch, unsigned* sig_ag,
                unsigned* const* peer_sig_ag, unsigned* done, unsigned done_base, int grid, int* err,
                cudaStream_t st) {
  RESIHP_CHECK(bytes % 16 == 0 && tp <= kMaxTp, "ag_publish: bad size or tp");
  PublishArgs a{};
  a.x = static_cast<const uint4*>(x);
  a.slot = static_cast<uint4*>(slot);
  a.nvec = bytes / 16;
  a.rank = rank;
  a.tp = tp;
  a.epoch = epoch;
  a.sig_ag = sig_ag;
  for (int p = 0; p < tp; ++p) a.peer_sig_ag[p] = peer_sig_ag[p];
  a.done = done;
  a.done_target = done_base + unsigned(grid);
  a.err = err;
  ag_publish_kernel<<<grid, 256, 0, st>>>(a);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

void ag_gemm(const void* x_local, const void* xg, const void* const* peer_x, const void* w, int64_t ldw, bool w_mn,
             void* y, int64_t ldy, int t_rows, int n, int k, int rank, int tp, unsigned epoch, unsigned* sig_ag,
             unsigned* ready, unsigned ready_base, int grid, int* err, cudaStream_t st) {
  RESIHP_CHECK(tp >= 2 && tp <= kMaxTp && t_rows % tp == 0 && (t_rows / tp) % kFBM == 0,
               "ag_gemm: rows per rank must be a multiple of 128");
  RESIHP_CHECK(n % 8 == 0 && k % 8 == 0, "ag_gemm: N and K must be multiples of 8");
  const int tl = t_rows / tp;
  const int bn = 256;
  CUtensorMap ta = make_tma_2d_bf16(x_local, tl, k, k, 64, kFBM);
  CUtensorMap ta2 = make_tma_2d_bf16(xg, t_rows, k, k, 64, kFBM);
  CUtensorMap tb = w_mn ? make_tma_2d_bf16(w, k, n, ldw, 64, 64) : make_tma_2d_bf16(w, n, k, ldw, 64, bn);
  FusedArgs g{};
  g.c = y;
  g.ldc = ldy;
  g.m = t_rows;
  g.n = n;
  g.k = k;
  g.err = err;
  CommArgs& c = g.comm;
  c.rank = rank;
  c.tp = tp;
  c.rows_per_rank = tl;
  c.epoch = epoch;
  for (int p = 0; p < tp; ++p) c.peer_x[p] = static_cast<const __nv_bfloat16*>(peer_x[p]);
  c.xg = static_cast<__nv_bfloat16*>(const_cast<void*>(xg));
  c.x_local = static_cast<const __nv_bfloat16*>(x_local);
  c.ldx = k;
  c.sig_ag = sig_ag;
  c.ready = ready;
  c.ready_target = ready_base + 2u * unsigned(grid);
  if (w_mn) launch_fused<256, true, 1>(ta, ta2, tb, g, grid, st);
  else launch_fused<256, false, 1>(ta, ta2, tb, g, grid, st);
}

void gemm_rs(const void* h, const void* w, int64_t ldw, bool w_mn, void* y_local, int64_t ldy, int t_rows, int n,
             int k, int rank, int tp, unsigned epoch, void* const* peer_recv, unsigned* const* peer_arrive,
             unsigned* const* peer_sig_rs, unsigned* arrive, unsigned* sig_rs, unsigned arrive_base,
             const void* recv_local, int grid, int* err, cudaStream_t st) {
  RESIHP_CHECK(tp >= 2 && tp <= kMaxTp && t_rows % tp == 0 && (t_rows / tp) % kFBM == 0,
               "gemm_rs: rows per rank must be a multiple of 128");
  RESIHP_CHECK(n % 32 == 0 && k % 8 == 0, "gemm_rs: N must be a multiple of 32 and K of 8");
  const int tl = t_rows / tp;
  const int bn = 256;
  CUtensorMap ta = make_tma_2d_bf16(h, t_rows, k, k, 64, kFBM);
  CUtensorMap tb = w_mn ? make_tma_2d_bf16(w, k, n, ldw, 64, 64) : make_tma_2d_bf16(w, n, k, ldw, 64, bn);
  FusedArgs g{};
  g.c = y_local;
  g.ldc = ldy;
  g.m = t_rows;
  g.n = n;
  g.k = k;
  g.err = err;
  CommArgs& c = g.comm;
  c.rank = rank;
  c.tp = tp;
  c.rows_per_rank = tl;
  c.epoch = epoch;
  for (int p = 0; p < tp; ++p) {
    c.peer_recv[p] = static_cast<__nv_bfloat16*>(peer_recv[p]);
    c.peer_arrive[p] = peer_arrive[p];
    c.peer_sig_rs[p] = peer_sig_rs[p];
  }
  c.arrive = arrive;
  c.sig_rs = sig_rs;
  c.recv_local = static_cast<__nv_bfloat16*>(const_cast<void*>(recv_local));
  const int tiles_per_chunk = (tl / kFBM) * ((n + bn - 1) / bn);
  c.arrive_target = arrive_base + 4u * unsigned(tiles_per_chunk);
  if (w_mn) launch_fused<256, true, 2>(ta, ta, tb, g, grid, st);
  else launch_fused<256, false, 2>(ta, ta, tb, g, grid, st);
}

// ---- symmetric workspace: CUDA IPC -------------------------------------------------------

void* symm_alloc(int64_t bytes, void* handle_out) {
  void* p = nullptr;
  RESIHP_CUDA_CHECK(cudaMalloc(&p, bytes));
  RESIHP_CUDA_CHECK(cudaMemset(p, 0, bytes));
  RESIHP_CUDA_CHECK(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), p));
  return p;
}

void* symm_open(const void* handle) {
  void* p = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  RESIHP_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return p;
}

void symm_close(void* p) { cudaIpcCloseMemHandle(p); }
void symm_free(void* p) { cudaFree(p); }

}  // namespace resihp
