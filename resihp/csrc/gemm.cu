// Persistent warp-specialised bf16 GEMM on the sm_100a tensor cores (tcgen05 + TMEM).
//
//   C[M,N] (=, +=) alpha * sum_k A(m,k) * B(n,k)      fp32 accumulation in TMEM
//
// Operands are read in place through TMA tensor maps, K-major or MN-major, so the
// three linear-layer products need no transposes:
//   forward  y  = x  w^T :  A = x  [M,K] K-major,        B = w [N,K] K-major
//   dgrad    dx = dy w   :  A = dy [M,N] K-major,        B = w [N,K] read N-major
//   wgrad    dw = dy^T x :  A = dy [M,N] read M-major,   B = x [M,K] read N-major
//
// One CTA per SM (persistent over output tiles, grouped along M for L2 reuse):
//   warp 0     TMA producer: fills a STAGES-deep ring of (A,B) 128B-swizzled smem tiles
//   warp 1     allocates TMEM; one lane issues tcgen05.mma (128 x BN x 16) into one of two
//              TMEM accumulators and commits each smem stage back to the producer
//   warps 2-5  epilogue: tcgen05.ld the finished accumulator (warp w owns TMEM lanes
//              32*(w%4)..+31 = tile rows), apply the epilogue, store to global memory;
//              the second accumulator lets the next tile's MMAs overlap this epilogue.
// Every barrier wait is bounded (common.cuh) and reports into ``err``.
//
// Replaces the reference's projections (``F.linear`` in resihp/parallel/tp.py:235-237,
// 243, 247-248, 272) and their autograd products.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "launch.h"

namespace resihp {

enum GemmEpilogue : int {
  kEpiStoreBf16 = 0,   // C(bf16) = alpha * acc
  kEpiStoreF32 = 1,    // C(f32)  = alpha * acc
  kEpiAccumF32 = 2,    // C(f32) += alpha * acc   (load, add, store)
  kEpiAddBf16 = 3,     // C(bf16) = alpha * acc + R(bf16)
  kEpiRedF32 = 4,      // C(f32) += alpha * acc   (red.global.add: no load latency in the epilogue)
};

// Fire-and-forget C[0..3] += v in L2. Every element of C is added to by exactly one
// thread of one CTA per launch, so the sum is the same single fp32 addition the
// load-add-store epilogue performs (atomic f32 adds flush subnormals to zero).
__device__ __forceinline__ void red_add_v4(float* p, float4 v) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

struct GemmArgs {
  void* c;
  const void* r;
  int64_t ldc;
  int64_t ldr;
  int m, n, k;
  float alpha;
  int* err;
};

constexpr int kBM = 128;
constexpr int kBK = 64;

template <int BN>
struct GemmShape {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kSmem = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int kTmemCols = 2 * BN;
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& tm, int& tn) {
  constexpr int kGroup = 8;
  const int per_group = kGroup * tiles_n;
  const int group = t / per_group;
  const int first = group * kGroup;
  const int size = min(tiles_m - first, kGroup);
  const int in_group = t % per_group;
  tm = first + in_group % size;
  tn = in_group / size;
}

// One thread's 32 consecutive accumulator columns (row ``row``, from column ``col0``)
// through the epilogue into C.
template <int EPI>
__device__ __forceinline__ void store_chunk(const GemmArgs& g, int row, int col0, const uint32_t (&v)[32]) {
  if (EPI == kEpiStoreBf16 || EPI == kEpiAddBf16) {
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(g.c) + int64_t(row) * g.ldc + col0;
    const __nv_bfloat16* res =
        EPI == kEpiAddBf16 ? static_cast<const __nv_bfloat16*>(g.r) + int64_t(row) * g.ldr + col0 : nullptr;
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (col0 + 8 * j >= g.n) break;
      float f[8];
      #pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = g.alpha * __uint_as_float(v[8 * j + e]);
      if (EPI == kEpiAddBf16) {
        uint4 rv = *reinterpret_cast<const uint4*>(res + 8 * j);
        const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rv);
        #pragma unroll
        for (int e = 0; e < 8; ++e) f[e] += __bfloat162float(rb[e]);
      }
      uint4 o;
      o.x = pack_bf16(f[0], f[1]);
      o.y = pack_bf16(f[2], f[3]);
      o.z = pack_bf16(f[4], f[5]);
      o.w = pack_bf16(f[6], f[7]);
      *reinterpret_cast<uint4*>(out + 8 * j) = o;
    }
  } else {
    float* out = static_cast<float*>(g.c) + int64_t(row) * g.ldc + col0;
    #pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (col0 + 4 * j >= g.n) break;
      float4 o = make_float4(g.alpha * __uint_as_float(v[4 * j]), g.alpha * __uint_as_float(v[4 * j + 1]),
                             g.alpha * __uint_as_float(v[4 * j + 2]), g.alpha * __uint_as_float(v[4 * j + 3]));
      if (EPI == kEpiRedF32) {
        red_add_v4(out + 4 * j, o);
        continue;
      }
      if (EPI == kEpiAccumF32) {
        float4 p = *reinterpret_cast<const float4*>(out + 4 * j);
        o.x += p.x; o.y += p.y; o.z += p.z; o.w += p.w;
      }
      *reinterpret_cast<float4*>(out + 4 * j) = o;
    }
  }
}

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, GemmArgs g) {
  pdl_enter();
  using S = GemmShape<BN>;
  constexpr int kStages = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * S::kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (g.m + kBM - 1) / kBM;
  const int tiles_n = (g.n + BN - 1) / BN;
  const int tiles = tiles_m * tiles_n;
  const int kblocks = (g.k + kBK - 1) / kBK;

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
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tma_a);
    tma_prefetch(&tma_b);
  }
  if (warp == 1) tmem_alloc(tmem_slot, S::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, tiles_m, tiles_n, tm, tn);
        const int m0 = tm * kBM, n0 = tn * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, g.err, kErrTmaWait)) { ok = false; break; }
          uint8_t* sa = smem + s * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_expect_tx(&full[s], S::kStageBytes);
          const int k0 = kb * kBK;
          if (A_MN) {
            tma_load_2d(sa, &tma_a, &full[s], m0, k0, g.err);
            tma_load_2d(sa + 8192, &tma_a, &full[s], m0 + 64, k0, g.err);
          } else {
            tma_load_2d(sa, &tma_a, &full[s], k0, m0, g.err);
          }
          if (B_MN) {
            #pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_2d(sb + c * 8192, &tma_b, &full[s], n0 + 64 * c, k0, g.err);
          } else {
            tma_load_2d(sb, &tma_b, &full[s], k0, n0, g.err);
          }
          if (++s == kStages) { s = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kBM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
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
        if (!tmem_span_ok(d, tmem_base, S::kTmemCols, BN, g.err)) break;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[s], ph, g.err, kErrMmaWait)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * S::kStageBytes);
          const uint32_t sb = sa + S::kABytes;
          #pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t da = A_MN ? smem_desc_sw128(sa + kk * 2048, 8192, 1024)
                                     : smem_desc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t db = B_MN ? smem_desc_sw128(sb + kk * 2048, 8192, 1024)
                                     : smem_desc_sw128(sb + kk * 32, 16, 1024);
            umma_bf16(d, da, db, idesc, (kb | kk) != 0);
          }
          umma_commit(&empty[s]);
          if (++s == kStages) { s = 0; ph ^= 1; }
        }
        umma_commit(&acc_full[a]);
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      int tm, tn;
      tile_coords(t, tiles_m, tiles_n, tm, tn);
      const int a = i & 1;
      const uint32_t accph = (i >> 1) & 1;
      if (!mbar_wait(&acc_full[a], accph, g.err, kErrEpiWait)) break;
      tc_fence_after();
      const int row = tm * kBM + q * 32 + lane;
      const bool row_ok = row < g.m;
      #pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        const uint32_t ta = tmem_base + a * BN + c * 32 + (uint32_t(q * 32) << 16);
        if (!tmem_span_ok(ta, tmem_base, S::kTmemCols, 32, g.err)) continue;
        tmem_ld32(ta, v);
        tmem_wait_ld();
        const int col0 = tn * BN + c * 32;
        if (!row_ok || col0 >= g.n) continue;
        store_chunk<EPI>(g, row, col0, v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------
// CTA-pair variant: 256 x 256 output tiles on two SMs (tcgen05 cta_group::2)
// ---------------------------------------------------------------------------------------
//
// A 2-CTA cluster computes one 256 x 256 tile per step: each CTA loads its own 128 rows
// of A and its own 128 rows (N) of B per K block, the leader's single MMA thread issues
// 256 x 256 x 16 pair MMAs that read both CTAs' halves, and each CTA's TMEM receives its
// 128 accumulator rows over all 256 columns. Per SM that is 32 KB of operand traffic per
// 128 x 256 x 64 of MMA work instead of 48 KB for the single-CTA 128 x 256 tile, which
// is what lets the tensor cores, not shared-memory / L2 bandwidth, set the pace.
//
//   both CTAs  warp 0     TMA producer for the CTA's halves; stage completion is counted
//                         on the leader's ``full`` barrier (the leader expects both halves)
//   leader     warp 1     pair MMAs; each stage is released to BOTH producers, each
//                         finished accumulator to BOTH epilogues (one commit per CTA)
//   both CTAs  warps 2-5  epilogue of the CTA's 128 rows; the accumulator is handed back
//                         on the leader's ``acc_empty`` (8 warp arrivals)
// No load is multicast: each CTA reads its own operand halves from this GPU's memory.

// Six 32 KB operand stages by default; seven still fit (7 x 32 KB + alignment slack and
// barriers = 230,656 of the 232,448 bytes a CTA may have), selected with
// RESIHP_GEMM_STAGES=7 (experimental: the extra stage covers more TMA latency).
constexpr int kPairStages = 6;

template <int STAGES>
struct PairShape {
  static constexpr int kABytes = 128 * kBK * 2;   // this CTA's 128 rows of A
  static constexpr int kBBytes = 128 * kBK * 2;   // this CTA's 128 rows (N) of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kSmem = STAGES * kStageBytes + 1024 + 256;
  static constexpr int kTmemCols = 512;           // two 256-column accumulators
  static_assert(kSmem <= 232448, "pair GEMM stages exceed the shared memory of a CTA");
  static_assert((2 * STAGES + 4) * 8 + 4 <= 256, "pair GEMM barriers exceed their area");
};

template <bool A_MN, bool B_MN, int EPI, int STAGES>
__global__ void __launch_bounds__(192, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, GemmArgs g) {
  pdl_enter();
  using S = PairShape<STAGES>;
  constexpr int kStages = STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * S::kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();  // 0: leader, 1: peer
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int tiles_m = (g.m + 255) / 256;
  const int tiles_n = (g.n + 255) / 256;
  const int tiles = tiles_m * tiles_n;
  const int kblocks = (g.k + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 8);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tma_a);
    tma_prefetch(&tma_b);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, S::kTmemCols);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += pairs) {
        int tm, tn;
        tile_coords(t, tiles_m, tiles_n, tm, tn);
        const int m0 = tm * 256 + int(cta) * 128, n0 = tn * 256 + int(cta) * 128;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, g.err, kErrTmaWait)) { ok = false; break; }
          uint8_t* sa = smem + s * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          if (cta == 0) mbar_expect_tx(&full[s], 2 * S::kStageBytes);  // both CTAs' halves
          const uint32_t bar = mapa_shared(&full[s], 0);
          const int k0 = kb * kBK;
          if (A_MN) {
            tma_load_2d_pair(sa, &tma_a, bar, m0, k0, g.err);
            tma_load_2d_pair(sa + 8192, &tma_a, bar, m0 + 64, k0, g.err);
          } else {
            tma_load_2d_pair(sa, &tma_a, bar, k0, m0, g.err);
          }
          if (B_MN) {
            tma_load_2d_pair(sb, &tma_b, bar, n0, k0, g.err);
            tma_load_2d_pair(sb + 8192, &tma_b, bar, n0 + 64, k0, g.err);
          } else {
            tma_load_2d_pair(sb, &tma_b, bar, k0, n0, g.err);
          }
          if (++s == kStages) { s = 0; ph ^= 1; }
        }
      }
      // Producer tail: wait until the leader has released every stage, so no pair-MMA
      // commit can arrive on this CTA's barriers after it exits.
      for (int j = 0; j < kStages && ok; ++j) {
        if (!mbar_wait(&empty[s], ph ^ 1, g.err, kErrTmaWait)) break;
        if (++s == kStages) { s = 0; ph ^= 1; }
      }
    }
  } else if (warp == 1) {
    if (cta == 0 && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(256, 256, A_MN ? 1 : 0, B_MN ? 1 : 0);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int i = 0;
      for (int t = pair; t < tiles && ok; t += pairs, ++i) {
        const int a = i & 1;
        const uint32_t accph = (i >> 1) & 1;
        if (!mbar_wait_cluster(&acc_empty[a], accph ^ 1, g.err, kErrMmaWait)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + a * 256;
        if (!tmem_span_ok(d, tmem_base, S::kTmemCols, 256, g.err)) break;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[s], ph, g.err, kErrMmaWait)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * S::kStageBytes);
          const uint32_t sb = sa + S::kABytes;
          #pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t da = A_MN ? smem_desc_sw128(sa + kk * 2048, 8192, 1024)
                                     : smem_desc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t db = B_MN ? smem_desc_sw128(sb + kk * 2048, 8192, 1024)
                                     : smem_desc_sw128(sb + kk * 32, 16, 1024);
            umma_bf16_pair(d, da, db, idesc, (kb | kk) != 0);
          }
          umma_commit_pair(smem_u32(&empty[s]));
          umma_commit_pair(mapa_shared(&empty[s], 1));
          if (++s == kStages) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&acc_full[a]));
        umma_commit_pair(mapa_shared(&acc_full[a], 1));
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t acc_empty_leader0 = mapa_shared(&acc_empty[0], 0);
    const uint32_t acc_empty_leader1 = mapa_shared(&acc_empty[1], 0);
    int i = 0;
    for (int t = pair; t < tiles; t += pairs, ++i) {
      int tm, tn;
      tile_coords(t, tiles_m, tiles_n, tm, tn);
      const int a = i & 1;
      const uint32_t accph = (i >> 1) & 1;
      if (!mbar_wait(&acc_full[a], accph, g.err, kErrEpiWait)) break;
      tc_fence_after();
      const int row = tm * 256 + int(cta) * 128 + q * 32 + lane;
      const bool row_ok = row < g.m;
      #pragma unroll 1
      for (int c = 0; c < 256 / 32; ++c) {
        uint32_t v[32];
        const uint32_t ta = tmem_base + a * 256 + c * 32 + (uint32_t(q * 32) << 16);
        if (!tmem_span_ok(ta, tmem_base, S::kTmemCols, 32, g.err)) continue;
        tmem_ld32(ta, v);
        tmem_wait_ld();
        const int col0 = tn * 256 + c * 32;
        if (!row_ok || col0 >= g.n) continue;
        store_chunk<EPI>(g, row, col0, v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(a == 0 ? acc_empty_leader0 : acc_empty_leader1);
    }
  }

  tc_fence_before();
  cluster_sync();  // no CTA leaves while its pair may still touch its barriers or TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, S::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult status;
    void* p = nullptr;
    RESIHP_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &status));
    RESIHP_CHECK(status == cudaDriverEntryPointSuccess && p != nullptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Row-major 2-D bf16 matrix [rows, cols] with row stride ``ld`` (elements), tiled by
// (box_cols, box_rows) with 128-byte swizzle. Out-of-range boxes read as zero.
CUtensorMap make_tma_2d_bf16(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_cols, int box_rows) {
  RESIHP_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  RESIHP_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  // The driver call needs this thread's context current; a thread whose first CUDA work
  // is this encode (e.g. an autograd worker served from the allocator cache) may not
  // have one yet, so make the current device's primary context current explicitly.
  int dev = 0;
  RESIHP_CUDA_CHECK(cudaGetDevice(&dev));
  RESIHP_CUDA_CHECK(cudaSetDevice(dev));
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  RESIHP_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", int(r));
  return map;
}

static int num_sms() {
  static int counts[64] = {0};
  int dev = 0;
  RESIHP_CUDA_CHECK(cudaGetDevice(&dev));
  if (counts[dev] == 0) RESIHP_CUDA_CHECK(cudaDeviceGetAttribute(&counts[dev], cudaDevAttrMultiProcessorCount, dev));
  return counts[dev];
}

template <int BN, bool A_MN, bool B_MN, int EPI>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g, cudaStream_t stream,
                        int max_ctas) {
  using S = GemmShape<BN>;
  auto kernel = gemm_kernel<BN, A_MN, B_MN, EPI>;
  static bool configured[64] = {false};
  int dev = 0;
  RESIHP_CUDA_CHECK(cudaGetDevice(&dev));
  if (!configured[dev]) {
    RESIHP_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem));
    configured[dev] = true;
  }
  const int tiles = ((g.m + kBM - 1) / kBM) * ((g.n + BN - 1) / BN);
  int grid = std::min(tiles, max_ctas > 0 ? max_ctas : num_sms());
  launch_pdl(kernel, grid, 192, S::kSmem, stream, ta, tb, g);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

// The operand-major / epilogue combinations the linear layers use:
//   forward  (K,K)   store bf16 or add residual
//   dgrad    (K,MN)  store bf16 or fp32
//   wgrad    (MN,MN) store or accumulate fp32 (load-add-store or red.global.add)
template <bool A_MN, bool B_MN, int EPI, int STAGES>
static void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g, cudaStream_t stream,
                        int max_ctas) {
  using S = PairShape<STAGES>;
  auto kernel = gemm_pair_kernel<A_MN, B_MN, EPI, STAGES>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // the kernel starts with pdl_enter()
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = S::kSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static int max_pairs[64] = {0};
  int dev = 0;
  RESIHP_CUDA_CHECK(cudaGetDevice(&dev));
  if (max_pairs[dev] == 0) {
    RESIHP_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem));
    cfg.gridDim = dim3(2, 1, 1);
    int n = 0;
    // pairs that can be resident at once (a persistent grid larger than that only queues)
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
      (void)cudaGetLastError();
      n = num_sms() / 2;
    }
    max_pairs[dev] = n;
  }
  const int tiles = ((g.m + 255) / 256) * ((g.n + 255) / 256);
  int pairs = std::min(tiles, max_pairs[dev]);
  if (max_ctas > 0) pairs = std::min(pairs, std::max(1, max_ctas / 2));
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  RESIHP_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, ta, tb, g));
}

// The same combinations on CTA pairs.
template <int ST>
static void dispatch_pair_stages(int epi, bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                                 const GemmArgs& g, cudaStream_t st, int max_ctas) {
  if (!a_mn && !b_mn && epi == kEpiStoreBf16) return launch_pair<false, false, kEpiStoreBf16, ST>(ta, tb, g, st, max_ctas);
  if (!a_mn && !b_mn && epi == kEpiAddBf16) return launch_pair<false, false, kEpiAddBf16, ST>(ta, tb, g, st, max_ctas);
  if (!a_mn && !b_mn && epi == kEpiStoreF32) return launch_pair<false, false, kEpiStoreF32, ST>(ta, tb, g, st, max_ctas);
  if (!a_mn && b_mn && epi == kEpiStoreBf16) return launch_pair<false, true, kEpiStoreBf16, ST>(ta, tb, g, st, max_ctas);
  if (!a_mn && b_mn && epi == kEpiStoreF32) return launch_pair<false, true, kEpiStoreF32, ST>(ta, tb, g, st, max_ctas);
  if (a_mn && b_mn && epi == kEpiStoreF32) return launch_pair<true, true, kEpiStoreF32, ST>(ta, tb, g, st, max_ctas);
  if (a_mn && b_mn && epi == kEpiAccumF32) return launch_pair<true, true, kEpiAccumF32, ST>(ta, tb, g, st, max_ctas);
  if (a_mn && b_mn && epi == kEpiRedF32) return launch_pair<true, true, kEpiRedF32, ST>(ta, tb, g, st, max_ctas);
  if (a_mn && b_mn && epi == kEpiStoreBf16) return launch_pair<true, true, kEpiStoreBf16, ST>(ta, tb, g, st, max_ctas);
  RESIHP_CHECK(false, "unsupported GEMM combination a_mn=", a_mn, " b_mn=", b_mn, " epi=", epi);
}

static int pair_stages() {
  static const int stages = [] {
    const char* v = std::getenv("RESIHP_GEMM_STAGES");
    return v != nullptr && std::strcmp(v, "7") == 0 ? 7 : kPairStages;
  }();
  return stages;
}

static void dispatch_pair(int epi, bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                          const GemmArgs& g, cudaStream_t st, int max_ctas) {
  if (pair_stages() == 7) return dispatch_pair_stages<7>(epi, a_mn, b_mn, ta, tb, g, st, max_ctas);
  return dispatch_pair_stages<kPairStages>(epi, a_mn, b_mn, ta, tb, g, st, max_ctas);
}

// CTA pairs for every GEMM that takes 256-column tiles (RESIHP_GEMM_PAIR=0: single CTAs).
static bool pair_enabled() {
  static int enabled = -1;
  if (enabled < 0) {
    const char* v = std::getenv("RESIHP_GEMM_PAIR");
    enabled = (v == nullptr || std::strcmp(v, "0") != 0) ? 1 : 0;
  }
  return enabled == 1;
}

template <int BN>
static void dispatch(int epi, bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g,
                     cudaStream_t st, int max_ctas) {
  if (!a_mn && !b_mn && epi == kEpiStoreBf16) return launch_gemm<BN, false, false, kEpiStoreBf16>(ta, tb, g, st, max_ctas);
  if (!a_mn && !b_mn && epi == kEpiAddBf16) return launch_gemm<BN, false, false, kEpiAddBf16>(ta, tb, g, st, max_ctas);
  if (!a_mn && !b_mn && epi == kEpiStoreF32) return launch_gemm<BN, false, false, kEpiStoreF32>(ta, tb, g, st, max_ctas);
  if (!a_mn && b_mn && epi == kEpiStoreBf16) return launch_gemm<BN, false, true, kEpiStoreBf16>(ta, tb, g, st, max_ctas);
  if (!a_mn && b_mn && epi == kEpiStoreF32) return launch_gemm<BN, false, true, kEpiStoreF32>(ta, tb, g, st, max_ctas);
  if (a_mn && b_mn && epi == kEpiStoreF32) return launch_gemm<BN, true, true, kEpiStoreF32>(ta, tb, g, st, max_ctas);
  if (a_mn && b_mn && epi == kEpiAccumF32) return launch_gemm<BN, true, true, kEpiAccumF32>(ta, tb, g, st, max_ctas);
  if (a_mn && b_mn && epi == kEpiRedF32) return launch_gemm<BN, true, true, kEpiRedF32>(ta, tb, g, st, max_ctas);
  if (a_mn && b_mn && epi == kEpiStoreBf16) return launch_gemm<BN, true, true, kEpiStoreBf16>(ta, tb, g, st, max_ctas);
  RESIHP_CHECK(false, "unsupported GEMM combination a_mn=", a_mn, " b_mn=", b_mn, " epi=", epi);
}

// Pick the N tile: 256 unless that leaves most SMs idle.
static int choose_bn(int m, int n) {
  if (n <= 128) return 128;
  const long tiles256 = long((m + kBM - 1) / kBM) * ((n + 255) / 256);
  return tiles256 < num_sms() ? 128 : 256;
}

void gemm_raw(const void* a, int64_t lda, bool a_mn, const void* b, int64_t ldb, bool b_mn, void* c, int64_t ldc,
              const void* r, int64_t ldr, int m, int n, int k, int epi, float alpha, int* err, cudaStream_t stream,
              int max_ctas, int force_bn) {
  RESIHP_CHECK(m > 0 && n > 0 && k > 0, "GEMM sizes must be positive");
  RESIHP_CHECK(n % 8 == 0, "GEMM needs N to be a multiple of 8 (16-byte output vectors)");
  RESIHP_CHECK(reinterpret_cast<uintptr_t>(c) % 16 == 0 && ldc % 8 == 0, "GEMM output must be 16-byte aligned");
  RESIHP_CHECK(force_bn == 0 || force_bn == 128 || force_bn == 256 || force_bn == 512,
               "force_bn must be 0, 128, 256 or 512 (CTA pairs)");
  int bn = force_bn ? force_bn : choose_bn(m, n);
  if (force_bn == 0 && n > 128 && m > kBM && pair_enabled()) {
    // CTA pairs whenever their 256 x 256 tiles fill the pairs about as evenly as the
    // single-CTA tiles fill the SMs (a pair tile runs ~5-10 % faster per FLOP)
    const int sms = num_sms(), pairs = sms / 2;
    const long tp = long((m + 255) / 256) * ((n + 255) / 256);
    const long ts = long((m + kBM - 1) / kBM) * ((n + bn - 1) / bn);
    const double fill_p = double(tp) / double(((tp + pairs - 1) / pairs) * pairs);
    const double fill_s = double(ts) / double(((ts + sms - 1) / sms) * sms);
    if (fill_p >= 0.9 * fill_s) bn = 512;
  }
  // A: K-major [m, k] (ld = lda) or M-major stored [k, m] (ld = lda). B boxes hold the
  // rows one CTA loads: the N tile, or its half on a CTA pair.
  CUtensorMap ta = a_mn ? make_tma_2d_bf16(a, k, m, lda, 64, 64) : make_tma_2d_bf16(a, m, k, lda, 64, kBM);
  CUtensorMap tb = b_mn ? make_tma_2d_bf16(b, k, n, ldb, 64, 64)
                        : make_tma_2d_bf16(b, n, k, ldb, 64, bn == 512 ? 128 : bn);
  GemmArgs g{c, r, ldc, ldr, m, n, k, alpha, err};
  if (bn == 512) return dispatch_pair(epi, a_mn, b_mn, ta, tb, g, stream, max_ctas);
  if (bn == 256) dispatch<256>(epi, a_mn, b_mn, ta, tb, g, stream, max_ctas);
  else dispatch<128>(epi, a_mn, b_mn, ta, tb, g, stream, max_ctas);
}

}  // namespace resihp
