// Causal flash attention (forward and backward) on the sm_100a tensor cores. Replaces the
// reference's materialised [B, H, S, S] scores, triu mask, softmax and weights @ v
// (resihp/parallel/tp.py:238-242, resihp/model.py:60-71).
//
// Q, K and V are read in place from the fused projection qkv[T, (Hq + 2*Hkv) * D]
// (row t = batch b, position t % S), GQA maps q head h to kv head h / (Hq / Hkv).
// One TMA tensor map (box 64 columns x 128 rows, 128-byte swizzle) serves every tile:
// a 64-column slab of 128 rows is a K-major operand when its columns are the reduction
// dimension (Q, K in S = Q K^T) and an MN-major operand when its rows are (V in P V).
//
// Forward, one CTA per (q block of 128 rows, q head, batch):
//   warp 0      TMA: Q once, then K_j / V_j into a 2-deep ring
//   warp 1      TMEM owner and MMA issuer: S_j = Q K_j^T into one of two TMEM S buffers,
//               O += P_j V_j into the TMEM O accumulator (S_{j+1} is issued before
//               PV_j so the tensor core works while softmax runs)
//   warps 2-9   softmax, two threads per query row (the two warps of a TMEM lane
//               quadrant take 64 columns each and exchange the row maximum through
//               shared memory): P = exp2(S * scale*log2e - m), P written back as packed
//               bf16 into its own S buffer in TMEM (the A operand of PV, read from
//               TMEM), each half of O rescaled in TMEM when the max grows (after the
//               previous PV), finally O / l stored as bf16 and the log-sum-exp kept.
// Backward (deterministic, no atomics):
//   attn_bwd_dkdv  one CTA per (kv block, kv head, batch), looping over every q head of
//                  the group and every causal q block: S^T = K Q^T, dP^T = V dO^T,
//                  P^T = exp(S^T - lse), dS^T = P^T (dP^T - Delta), then
//                  dV += P^T dO and dK += dS^T Q accumulated in TMEM.
//   attn_bwd_dq    one CTA per (q block, q head, batch): S, dP recomputed, dQ += dS K.
//   Both run the kv (dK/dV) or q (dQ) side in sub-blocks of 64 rows with double-buffered
//   TMEM scores and eight elementwise warps (see the kernels).
//   P^T / dS^T (and dS in the dQ kernel) go back into their score buffers in TMEM as
//   packed bf16 and are the A operands of the dV / dK (dQ) MMAs, read from TMEM.
// All waits are bounded (common.cuh) and report into the error word.
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "launch.h"

namespace resihp {

namespace {

constexpr int kBlk = 128;          // q rows and kv rows per tile
constexpr float kLog2e = 1.4426950408889634f;

struct AttnArgs {
  __nv_bfloat16* out;      // [T, Hq*D] (forward) or dqkv [T, W] (backward)
  float* lse;              // [B, Hq, S] natural-log log-sum-exp
  const __nv_bfloat16* dout;  // backward: dO [T, Hq*D]
  const float* delta;      // backward: rowsum(dO * O) [B, Hq, S]
  int seq, hq, hkv, d;
  int64_t out_ld;
  int64_t dout_ld;
  float scale;             // 1/sqrt(D)
  int* err;
};

// 2^x with the hardware approximation (one MUFU instruction; relative error ~2^-22,
// far below the bf16 rounding P and dS go through next).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Row ``r`` of 64-column chunk ``chunk`` of a K-major 128B-swizzled bf16 tile with
// ``rows`` rows (TMA layout: 16-byte unit u of row r sits at unit u ^ (r & 7)) into 32
// TMEM columns at ``taddr`` (this warp's lanes), as packed bf16 pairs in column order:
// the layout of an MMA A operand read from tensor memory.
__device__ __forceinline__ void sw128_row_to_tmem(const uint8_t* tile, int rows, int chunk, int r, uint32_t taddr) {
  const uint8_t* row = tile + (chunk * rows + r) * 128;
  uint32_t w[32];
  #pragma unroll
  for (int u = 0; u < 8; ++u) {
    const uint4 v = *reinterpret_cast<const uint4*>(row + ((u ^ (r & 7)) * 16));
    w[4 * u] = v.x;
    w[4 * u + 1] = v.y;
    w[4 * u + 2] = v.z;
    w[4 * u + 3] = v.w;
  }
  tmem_st16(taddr, *reinterpret_cast<const uint32_t(*)[16]>(w));
  tmem_st16(taddr + 16, *reinterpret_cast<const uint32_t(*)[16]>(w + 16));
}

constexpr int kFwdThreads = 64 + 8 * 32;  // producer, MMA issuer, eight softmax warps

template <int D>
struct FwdSmem {
  static constexpr int kQ = kBlk * D * 2;
  static constexpr int kKV = kBlk * D * 2;
  static constexpr int kStages = 2;
  static constexpr int kMx = 6 * kBlk * 4;   // row-max exchange [2 blocks][2 halves][128], row-sum [2][128]
  static constexpr int kBytes = kQ + 2 * kStages * kKV + kMx + 1024 + 256;
};

template <int D>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm, AttnArgs a) {
  pdl_enter();
  using L = FwdSmem<D>;
  constexpr int ST = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
  uint8_t* sq = smem;
  uint8_t* sk = sq + L::kQ;                 // ST stages of K
  uint8_t* sv = sk + ST * L::kKV;           // ST stages of V
  float* s_mx = reinterpret_cast<float*>(sv + ST * L::kKV);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sv + ST * L::kKV + L::kMx);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + ST;
  uint64_t* k_empty = v_full + ST;   // K of a stage read by its S MMAs (refilled a step before V)
  uint64_t* v_empty = k_empty + ST;  // V of a stage read by its PV MMAs
  uint64_t* s_full = v_empty + ST;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* pv_done = p_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 1);

  // CTAs are dispatched in linear order with x fastest: the causal block is the slowest
  // grid dimension, so every (head, batch) pair's longest block goes first (longest
  // processing time first keeps the last wave short)
  const int qblk = (a.seq / kBlk) - 1 - blockIdx.z;
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const int kvh = h / (a.hq / a.hkv);
  const int nblk = qblk + 1;
  const int row0 = b * a.seq + qblk * kBlk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 8);
    }
    mbar_init(p_full, 8);
    mbar_init(pv_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_o = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch(&tm);
      mbar_expect_tx(q_full, L::kQ);
      #pragma unroll
      for (int c = 0; c < D / 64; ++c) tma_load_2d(sq + c * kBlk * 128, &tm, q_full, h * D + 64 * c, row0, a.err);
      // K runs one block ahead of V: K_j as soon as S_{j-ST} has read its stage, then
      // V_{j-1} once PV_{j-1-ST} has read its stage
      for (int j = 0; j <= nblk; ++j) {
        if (j < nblk) {
          const int st = j % ST;
          if (!mbar_wait(&k_empty[st], ((j / ST) & 1) ^ 1, a.err, kErrTmaWait)) break;
          mbar_expect_tx(&k_full[st], L::kKV);
          #pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_2d(sk + st * L::kKV + c * kBlk * 128, &tm, &k_full[st], (a.hq + kvh) * D + 64 * c,
                        b * a.seq + j * kBlk, a.err);
        }
        if (j >= 1) {
          const int jv = j - 1;
          const int st = jv % ST;
          if (!mbar_wait(&v_empty[st], ((jv / ST) & 1) ^ 1, a.err, kErrTmaWait)) break;
          mbar_expect_tx(&v_full[st], L::kKV);
          #pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_2d(sv + st * L::kKV + c * kBlk * 128, &tm, &v_full[st], (a.hq + a.hkv + kvh) * D + 64 * c,
                        b * a.seq + jv * kBlk, a.err);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16_f32(kBlk, kBlk, 0, 0);
      constexpr uint32_t id_o = idesc_bf16_f32(kBlk, D, 0, 1);
      const uint32_t q_addr = smem_u32(sq);
      bool ok = mbar_wait(q_full, 0, a.err, kErrMmaWait);
      auto issue_pv = [&](int j) -> bool {
        const int st = j % ST;
        if (!mbar_wait(p_full, j & 1, a.err, kErrMmaWait)) return false;
        if (!mbar_wait(&v_full[st], (j / ST) & 1, a.err, kErrMmaWait)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sv + st * L::kKV);
        #pragma unroll
        for (int kk = 0; kk < kBlk / 16; ++kk) {
          // A = P of block j from TMEM: packed bf16 in the first 32 columns of each
          // 64-column half of S buffer j & 1 (8 columns per 16 kv)
          const uint32_t pa = tmem + uint32_t((j & 1) * kBlk + (kk >> 2) * (kBlk / 2) + (kk & 3) * 8);
          const uint64_t db = smem_desc_sw128(v_addr + kk * 2048, kBlk * 128, 1024);
          umma_bf16_ts(t_o, pa, db, id_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(pv_done);
        umma_commit(&v_empty[st]);
        return true;
      };
      for (int j = 0; j < nblk && ok; ++j) {
        const int st = j % ST;
        const int sb = j & 1;
        if (!mbar_wait(&k_full[st], (j / ST) & 1, a.err, kErrMmaWait)) { ok = false; break; }
        if (!mbar_wait(&s_empty[sb], ((j >> 1) & 1) ^ 1, a.err, kErrMmaWait)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sk + st * L::kKV);
        #pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kBlk * 128 + (kk & 3) * 32;
          umma_bf16(tmem + sb * kBlk, smem_desc_sw128(q_addr + off, 16, 1024),
                    smem_desc_sw128(k_addr + off, 16, 1024), id_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[st]);
        if (j > 0 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) issue_pv(nblk - 1);
    }
  } else {
    // eight softmax warps: the two warps of a TMEM lane quadrant split each row's 128
    // columns (and O's D columns); only the row maximum is exchanged per block
    const int q4 = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = q4 * 32 + lane;           // query row within the tile
    const uint32_t lane_off = uint32_t(q4 * 32) << 16;
    const float sl2 = a.scale * kLog2e;
    constexpr int kHalf = kBlk / 2;
    float m = -INFINITY, l = 0.f;           // l: this half's share of the row sum
    bool ok = true;
    // Every softmax thread passes named barrier 2 exactly once per block and once after
    // the loop, also after a wait ran out (it then only keeps the barrier count), so the
    // two warps of a pair can never wait at different barrier instances.
    for (int j = 0; j < nblk; ++j) {
      const int sb = j & 1;
      if (ok && !mbar_wait(&s_full[sb], (j >> 1) & 1, a.err, kErrEpiWait)) ok = false;
      const bool diag = j == qblk;
      uint32_t v[kHalf];
      float mloc = -INFINITY;
      if (ok) {
        tc_fence_after();
        const uint32_t t_s = tmem + sb * kBlk + lane_off + half * kHalf;
        #pragma unroll
        for (int c = 0; c < kHalf; c += 32) tmem_ld32(t_s + c, *reinterpret_cast<uint32_t(*)[32]>(v + c));
        tmem_wait_ld();
        if (diag) {
          #pragma unroll
          for (int e = 0; e < kHalf; ++e)
            if (half * kHalf + e <= r) mloc = fmaxf(mloc, __uint_as_float(v[e]));
        } else {
          #pragma unroll
          for (int e = 0; e < kHalf; ++e) mloc = fmaxf(mloc, __uint_as_float(v[e]));
        }
      }
      s_mx[(sb * 2 + half) * kBlk + r] = mloc;
      asm volatile("bar.sync 2, 256;" ::: "memory");
      if (!ok) continue;
      const float mx = fmaxf(m, fmaxf(mloc, s_mx[(sb * 2 + (half ^ 1)) * kBlk + r]));
      const float alpha = fast_exp2((m - mx) * sl2);   // 0 on the first block (m = -inf)
      const float neg = mx * sl2;
      // P goes into this block's own S buffer in TMEM, so it does not wait for PV_{j-1}
      float rowsum = 0.f;
      #pragma unroll
      for (int c = 0; c < kHalf; c += 32) {
        uint32_t pk[16];
        #pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int col = half * kHalf + c + e;
          float p0 = fast_exp2(fmaf(__uint_as_float(v[c + e]), sl2, -neg));
          float p1 = fast_exp2(fmaf(__uint_as_float(v[c + e + 1]), sl2, -neg));
          if (diag && col > r) p0 = 0.f;
          if (diag && col + 1 > r) p1 = 0.f;
          rowsum += p0 + p1;
          pk[e / 2] = pack_bf16(p0, p1);
        }
        // packed P over the S values this warp already holds in registers: the first 32
        // columns of its 64-column half, the A operand of PV_j
        tmem_st16(tmem + sb * kBlk + lane_off + half * kHalf + c / 2, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);
      l = l * alpha + rowsum;
      m = mx;
      // rescale this half's columns of the running O when this warp saw the max grow
      // (after PV_{j-1}, which accumulates into O, has completed)
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        if (!mbar_wait(pv_done, (j - 1) & 1, a.err, kErrEpiWait)) { ok = false; continue; }
        tc_fence_after();
        #pragma unroll 1
        for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 16) {
          uint32_t w16[16];
          tmem_ld16(t_o + lane_off + c, w16);
          tmem_wait_ld();
          #pragma unroll
          for (int e = 0; e < 16; ++e) w16[e] = __float_as_uint(__uint_as_float(w16[e]) * alpha);
          tmem_st16(t_o + lane_off + c, w16);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // the row sum: both halves' shares, added in half order (own slots: the partner may
    // still be reading the last block's maximum)
    s_mx[(4 + half) * kBlk + r] = l;
    asm volatile("bar.sync 2, 256;" ::: "memory");
    const float lsum = s_mx[4 * kBlk + r] + s_mx[5 * kBlk + r];
    if (ok && mbar_wait(pv_done, (nblk - 1) & 1, a.err, kErrEpiWait)) {
      tc_fence_after();
      const float inv = 1.f / lsum;
      __nv_bfloat16* dst = a.out + int64_t(row0 + r) * a.out_ld + int64_t(h) * D;
      #pragma unroll 1
      for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 32) {
        uint32_t w32[32];
        tmem_ld32(t_o + lane_off + c, w32);
        tmem_wait_ld();
        #pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 o;
          o.x = pack_bf16(__uint_as_float(w32[8 * u + 0]) * inv, __uint_as_float(w32[8 * u + 1]) * inv);
          o.y = pack_bf16(__uint_as_float(w32[8 * u + 2]) * inv, __uint_as_float(w32[8 * u + 3]) * inv);
          o.z = pack_bf16(__uint_as_float(w32[8 * u + 4]) * inv, __uint_as_float(w32[8 * u + 5]) * inv);
          o.w = pack_bf16(__uint_as_float(w32[8 * u + 6]) * inv, __uint_as_float(w32[8 * u + 7]) * inv);
          *reinterpret_cast<uint4*>(dst + c + 8 * u) = o;
        }
      }
      if (half == 0) a.lse[(int64_t(b) * a.hq + h) * a.seq + qblk * kBlk + r] = m * a.scale + logf(lsum);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Delta[b, h, s] = sum_d dO * O  (fp32)
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ o, int64_t o_ld, const __nv_bfloat16* __restrict__ dout,
                                  int64_t do_ld, float* __restrict__ delta, int rows, int seq, int hq, int d) {
  pdl_enter();
  // eight lanes per (token, head): 16-byte loads, a three-step shuffle reduction
  const int lane = threadIdx.x & 31;
  const int idx = ((blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 4 + (lane >> 3);
  const int gl = lane & 7;
  const bool live = idx < rows * hq;
  float acc = 0.f;
  int t = 0, h = 0;
  if (live) {
    t = idx / hq;
    h = idx % hq;
    const __nv_bfloat16* po = o + int64_t(t) * o_ld + int64_t(h) * d;
    const __nv_bfloat16* pd = dout + int64_t(t) * do_ld + int64_t(h) * d;
    for (int c = gl * 8; c < d; c += 64) {
      const uint4 xr = *reinterpret_cast<const uint4*>(po + c);
      const uint4 yr = *reinterpret_cast<const uint4*>(pd + c);
      const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&xr);
      const __nv_bfloat162* y = reinterpret_cast<const __nv_bfloat162*>(&yr);
      #pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 a = __bfloat1622float2(x[e]), b = __bfloat1622float2(y[e]);
        acc += a.x * b.x + a.y * b.y;
      }
    }
  }
  #pragma unroll
  for (int off = 4; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (live && gl == 0) {
    const int b = t / seq, s = t % seq;
    delta[(int64_t(b) * hq + h) * seq + s] = acc;
  }
}

// ---- backward: dK, dV ----------------------------------------------------------------
//
// One CTA per (kv block of 128 rows, kv head, batch), looping over every q head of the
// group and every causal q sub-block of 64 rows. Sixty-four q rows per step keep
// S^T / dP^T small enough (2 x 64 TMEM columns each) to double-buffer next to the dV and
// dK accumulators; Q / dO / lse / delta come through a three-stage ring (their loads run
// two steps ahead, off the critical path) and P^T / dS^T go back into the step's TMEM
// score buffers, so step i+1's S^T and dP^T MMAs run while the elementwise warps turn
// step i into P^T and dS^T, and step i's dV / dK MMAs run while they do step i+1:
//   warp 0      TMA: K, V once; then Q_i, dO_i (64 rows) and their lse / delta rows
//   warp 1      MMA: S^T_i = K Q_i^T, dP^T_i = V dO_i^T (128 x 64), then dV += P^T_{i-1} dO_{i-1},
//               dK += dS^T_{i-1} Q_{i-1} (128 x D)
//   warps 2-9   elementwise, two warps per TMEM lane quadrant (32 q columns each):
//               P^T = exp2(S^T * scale*log2e - lse*log2e) (causal mask on the diagonal),
//               dS^T = P^T (dP^T - Delta), both as packed bf16 into TMEM.
constexpr int kQs = 64;             // q rows per dK/dV step
constexpr int kQdStages = 3;        // Q / dO / lse / delta ring: loads run two steps ahead
constexpr int kEwWarps = 8;         // elementwise warps
constexpr int kDkdvThreads = 64 + 32 * kEwWarps;

template <int D>
struct DkdvSmem {
  static constexpr int kKV = kBlk * D * 2;   // K or V tile
  static constexpr int kQ = kQs * D * 2;     // one Q or dO tile of 64 rows
  static constexpr int kBytes = 2 * kKV + 2 * kQdStages * kQ + 2 * kQdStages * kQs * 4 + 1024 + 256;
};


template <int D>
__global__ void __launch_bounds__(kDkdvThreads, 1)
    attn_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_do, AttnArgs a) {
  pdl_enter();
  using L = DkdvSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
  uint8_t* sk = smem;
  uint8_t* sv = sk + L::kKV;
  constexpr int QS = kQdStages;
  uint8_t* sq = sv + L::kKV;          // QS stages
  uint8_t* sdo = sq + QS * L::kQ;     // QS stages
  float* s_lse = reinterpret_cast<float*>(sdo + QS * L::kQ);  // [QS][kQs]
  float* s_delta = s_lse + QS * kQs;                            // [QS][kQs]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_delta + QS * kQs);
  uint64_t* kv_full = bars;
  uint64_t* qd_full = bars + 1;          // [QS] Q, dO, lse, delta of a step landed
  uint64_t* qd_empty = qd_full + QS;     // [QS] the dV/dK MMAs reading that step's Q, dO are done
  uint64_t* st_full = qd_empty + QS;     // [2] S^T, dP^T of a step in TMEM
  uint64_t* st_empty = st_full + 2;      // [2] the elementwise warps read them
  uint64_t* ds_full = st_empty + 2;      // [2] P^T, dS^T of a step back in TMEM
  uint64_t* acc_done = ds_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_done + 1);

  const int kvblk = blockIdx.z;  // slowest grid dimension: the longest causal ranges go first
  const int g = blockIdx.x;
  const int b = blockIdx.y;
  const int group = a.hq / a.hkv;
  const int nq = a.seq / kQs - 2 * kvblk;  // causal: q sub-blocks 2*kvblk .. end
  const int steps = nq * group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kv_row0 = b * a.seq + kvblk * kBlk;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < QS; ++s) {
      mbar_init(&qd_full[s], 1);
      mbar_init(&qd_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&st_full[s], 1);
      mbar_init(&st_empty[s], kEwWarps);
      mbar_init(&ds_full[s], kEwWarps);
    }
    mbar_init(acc_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S^T[2] 0 / 64, dP^T[2] 128 / 192, dV 256.., dK 256+D..
  const uint32_t t_dv = tmem + 256, t_dk = tmem + 256 + D;

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(kv_full, 2 * L::kKV);
      #pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_2d(sk + c * kBlk * 128, &tm_kv, kv_full, (a.hq + g) * D + 64 * c, kv_row0, a.err);
        tma_load_2d(sv + c * kBlk * 128, &tm_kv, kv_full, (a.hq + a.hkv + g) * D + 64 * c, kv_row0, a.err);
      }
      for (int it = 0; it < steps; ++it) {
        const int s = it % QS;
        if (!mbar_wait(&qd_empty[s], ((it / QS) & 1) ^ 1, a.err, kErrTmaWait)) break;
        const int h = g * group + it / nq;
        const int qs = 2 * kvblk + it % nq;
        const int q_row0 = b * a.seq + qs * kQs;
        const int64_t stat = (int64_t(b) * a.hq + h) * a.seq + qs * kQs;
        mbar_expect_tx(&qd_full[s], 2 * L::kQ + 2 * kQs * 4);
        #pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_2d(sq + s * L::kQ + c * kQs * 128, &tm_q, &qd_full[s], h * D + 64 * c, q_row0, a.err);
          tma_load_2d(sdo + s * L::kQ + c * kQs * 128, &tm_do, &qd_full[s], h * D + 64 * c, q_row0, a.err);
        }
        bulk_load(s_lse + s * kQs, a.lse + stat, kQs * 4, &qd_full[s]);
        bulk_load(s_delta + s * kQs, a.delta + stat, kQs * 4, &qd_full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16_f32(kBlk, kQs, 0, 0);
      constexpr uint32_t id_acc = idesc_bf16_f32(kBlk, D, 0, 1);
      const uint32_t k_addr = smem_u32(sk), v_addr = smem_u32(sv);
      bool ok = mbar_wait(kv_full, 0, a.err, kErrMmaWait);
      for (int it = 0; it <= steps && ok; ++it) {
        if (it < steps) {
          const int s = it & 1;
          const int s3 = it % QS;
          if (!mbar_wait(&qd_full[s3], (it / QS) & 1, a.err, kErrMmaWait)) { ok = false; break; }
          if (!mbar_wait(&st_empty[s], ((it >> 1) & 1) ^ 1, a.err, kErrMmaWait)) { ok = false; break; }
          tc_fence_after();
          const uint32_t q_addr = smem_u32(sq + s3 * L::kQ), do_addr = smem_u32(sdo + s3 * L::kQ);
          #pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t okv = (kk >> 2) * kBlk * 128 + (kk & 3) * 32;
            const uint32_t oq = (kk >> 2) * kQs * 128 + (kk & 3) * 32;
            umma_bf16(tmem + s * kQs, smem_desc_sw128(k_addr + okv, 16, 1024), smem_desc_sw128(q_addr + oq, 16, 1024),
                      id_s, kk > 0);
            umma_bf16(tmem + 128 + s * kQs, smem_desc_sw128(v_addr + okv, 16, 1024),
                      smem_desc_sw128(do_addr + oq, 16, 1024), id_s, kk > 0);
          }
          umma_commit(&st_full[s]);
        }
        if (it >= 1) {
          const int p = it - 1;
          const int sp = p & 1;
          if (!mbar_wait(&ds_full[sp], (p >> 1) & 1, a.err, kErrMmaWait)) { ok = false; break; }
          tc_fence_after();
          const int sp3 = p % QS;
          const uint32_t q_addr = smem_u32(sq + sp3 * L::kQ), do_addr = smem_u32(sdo + sp3 * L::kQ);
          #pragma unroll
          for (int kk = 0; kk < kQs / 16; ++kk) {
            // A from TMEM: P^T / dS^T as packed bf16 pairs, 16 q columns = 8 TMEM columns
            // per K step; the two 32-column halves sit at the start of each half's region
            const uint32_t acol = uint32_t(sp * kQs + (kk >> 1) * 32 + (kk & 1) * 8);
            umma_bf16_ts(t_dv, tmem + acol, smem_desc_sw128(do_addr + kk * 2048, kQs * 128, 1024), id_acc,
                         (p > 0 || kk > 0));
            umma_bf16_ts(t_dk, tmem + 128 + acol, smem_desc_sw128(q_addr + kk * 2048, kQs * 128, 1024), id_acc,
                         (p > 0 || kk > 0));
          }
          umma_commit(&qd_empty[sp3]);
        }
      }
      if (ok) umma_commit(acc_done);
    }
  } else {
    const int quad = warp & 3;                 // TMEM lane quadrant
    const int half = (warp - 2) >> 2;          // which 32 of the 64 q columns
    const int c_row = quad * 32 + lane;        // kv row within the tile
    const int k_pos = kvblk * kBlk + c_row;    // its position in the sequence
    const uint32_t lane_off = uint32_t(quad * 32) << 16;
    const float sl2 = a.scale * kLog2e;
    bool ok = true;
    for (int it = 0; it < steps; ++it) {
      const int s = it & 1;
      const uint32_t n = (it >> 1) & 1;
      const int qs = 2 * kvblk + it % nq;
      const bool diag = qs < 2 * kvblk + 2;   // q sub-block overlaps the kv block: causal mask
      if (!mbar_wait(&st_full[s], n, a.err, kErrEpiWait)) { ok = false; break; }
      tc_fence_after();
      uint32_t sv32[32], dv32[32];
      tmem_ld32(tmem + s * kQs + lane_off + half * 32, sv32);
      tmem_ld32(tmem + 128 + s * kQs + lane_off + half * 32, dv32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&st_empty[s]);
      // lse / delta of this step landed with Q (the MMA that filled S^T waited for them)
      const int s3 = it % QS;
      if (!mbar_wait(&qd_full[s3], (it / QS) & 1, a.err, kErrEpiWait)) { ok = false; break; }
      const float* lse = s_lse + s3 * kQs + half * 32;
      const float* dlt = s_delta + s3 * kQs + half * 32;
      const int q_pos0 = qs * kQs + half * 32;
      uint32_t pk[16], dk[16];
      #pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float p[2], ds[2];
        #pragma unroll
        for (int z = 0; z < 2; ++z) {
          float pv = fast_exp2(fmaf(__uint_as_float(sv32[e + z]), sl2, -lse[e + z] * kLog2e));
          if (diag && q_pos0 + e + z < k_pos) pv = 0.f;
          p[z] = pv;
          ds[z] = pv * (__uint_as_float(dv32[e + z]) - dlt[e + z]);
        }
        pk[e / 2] = pack_bf16(p[0], p[1]);
        dk[e / 2] = pack_bf16(ds[0], ds[1]);
      }
      // P^T and dS^T back into this step's S^T / dP^T TMEM buffers (the first 16 columns
      // of this warp's 32): the A operands of the dV / dK MMAs. The buffers are free: the
      // MMAs that read the previous step of this parity were issued (in order) before the
      // ones that filled S^T here, and the next MMAs that write them are issued after
      // this step's dV / dK MMAs.
      tmem_st16(tmem + s * kQs + lane_off + half * 32, pk);
      tmem_st16(tmem + 128 + s * kQs + lane_off + half * 32, dk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[s]);
    }
    if (ok && steps > 0 && mbar_wait(acc_done, 0, a.err, kErrEpiWait)) {
      tc_fence_after();
      __nv_bfloat16* dk_dst = a.out + int64_t(kv_row0 + c_row) * a.out_ld + int64_t(a.hq + g) * D;
      __nv_bfloat16* dv_dst = a.out + int64_t(kv_row0 + c_row) * a.out_ld + int64_t(a.hq + a.hkv + g) * D;
      #pragma unroll 1
      for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 32) {
        uint32_t v1[32], v2[32];
        tmem_ld32(t_dv + lane_off + c, v1);
        tmem_ld32(t_dk + lane_off + c, v2);
        tmem_wait_ld();
        #pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 o1, o2;
          o1.x = pack_bf16(__uint_as_float(v1[8 * u + 0]), __uint_as_float(v1[8 * u + 1]));
          o1.y = pack_bf16(__uint_as_float(v1[8 * u + 2]), __uint_as_float(v1[8 * u + 3]));
          o1.z = pack_bf16(__uint_as_float(v1[8 * u + 4]), __uint_as_float(v1[8 * u + 5]));
          o1.w = pack_bf16(__uint_as_float(v1[8 * u + 6]), __uint_as_float(v1[8 * u + 7]));
          o2.x = pack_bf16(__uint_as_float(v2[8 * u + 0]) * a.scale, __uint_as_float(v2[8 * u + 1]) * a.scale);
          o2.y = pack_bf16(__uint_as_float(v2[8 * u + 2]) * a.scale, __uint_as_float(v2[8 * u + 3]) * a.scale);
          o2.z = pack_bf16(__uint_as_float(v2[8 * u + 4]) * a.scale, __uint_as_float(v2[8 * u + 5]) * a.scale);
          o2.w = pack_bf16(__uint_as_float(v2[8 * u + 6]) * a.scale, __uint_as_float(v2[8 * u + 7]) * a.scale);
          *reinterpret_cast<uint4*>(dv_dst + c + 8 * u) = o1;
          *reinterpret_cast<uint4*>(dk_dst + c + 8 * u) = o2;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---- backward: dQ --------------------------------------------------------------------
//
// One CTA per (q block of 128 rows, q head, batch), looping over the causal kv range in
// sub-blocks of 64 rows, mirroring the dK/dV kernel: S_j / dP_j (128 x 64) double-buffered
// in TMEM next to the dQ accumulator, K_j / V_j in a three-stage ring and dS written back
// into the sub-block's S buffer, so the MMAs of one sub-block overlap the elementwise
// work of the previous one:
//   warp 0      TMA: Q, dO once; K_j, V_j (64 rows) into the ring
//   warp 1      MMA: S_j = Q K_j^T, dP_j = dO V_j^T, then dQ += dS_{j-1} K_{j-1}
//   warps 2-9   elementwise, two warps per TMEM lane quadrant (32 kv columns each):
//               dS = P (dP - Delta), P = exp2(S * scale*log2e - lse*log2e), causal mask.
constexpr int kKs = 64;   // kv rows per dQ step
constexpr int kDqStages = 3;

template <int D>
struct DqSmem {
  static constexpr int kT = kBlk * D * 2;    // Q or dO tile
  static constexpr int kKV = kKs * D * 2;    // one K or V tile of 64 rows
  static constexpr int kBytes = 2 * kT + 2 * kDqStages * kKV + 1024 + 256;
};

template <int D>
__global__ void __launch_bounds__(kDkdvThreads, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tm, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_kv64, AttnArgs a) {
  pdl_enter();
  using L = DqSmem<D>;
  constexpr int ST = kDqStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
  uint8_t* sq = smem;
  uint8_t* sdo = sq + L::kT;
  uint8_t* sk = sdo + L::kT;           // ST stages
  uint8_t* sv = sk + ST * L::kKV;      // ST stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(sv + ST * L::kKV);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;              // [ST]
  uint64_t* kv_empty = kv_full + ST;         // [ST]
  uint64_t* s_full = kv_empty + ST;          // [2] S, dP of a sub-block in TMEM
  uint64_t* s_empty = s_full + 2;            // [2] the elementwise warps read them
  uint64_t* ds_full = s_empty + 2;           // [2] dS of a sub-block back in TMEM
  uint64_t* dq_done = ds_full + 2;
  uint64_t* qo_tmem = dq_done + 1;           // Q and dO copied into TMEM (the S / dP A operands)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qo_tmem + 1);

  const int qblk = (a.seq / kBlk) - 1 - blockIdx.z;   // slowest grid dimension: heaviest first
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const int kvh = h / (a.hq / a.hkv);
  const int nkv = 2 * qblk + 2;                       // kv sub-blocks 0 .. 2*qblk+1
  const int row0 = b * a.seq + qblk * kBlk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], kEwWarps);
      mbar_init(&ds_full[s], kEwWarps);
    }
    mbar_init(dq_done, 1);
    mbar_init(qo_tmem, kEwWarps);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S[2] 0 / 64, dP[2] 128 / 192, dQ 256..383, Q 384..447, dO 448..511
  // (Q and dO as packed bf16: the A operands of every S and dP MMA, read from TMEM
  // instead of shared memory)
  const uint32_t t_dq = tmem + 256, t_q = tmem + 384, t_do = tmem + 448;

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(q_full, 2 * L::kT);
      #pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_2d(sq + c * kBlk * 128, &tm, q_full, h * D + 64 * c, row0, a.err);
        tma_load_2d(sdo + c * kBlk * 128, &tm_do, q_full, h * D + 64 * c, row0, a.err);
      }
      for (int j = 0; j < nkv; ++j) {
        const int st = j % ST;
        if (!mbar_wait(&kv_empty[st], ((j / ST) & 1) ^ 1, a.err, kErrTmaWait)) break;
        const int kv_row = b * a.seq + j * kKs;
        mbar_expect_tx(&kv_full[st], 2 * L::kKV);
        #pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_2d(sk + st * L::kKV + c * kKs * 128, &tm_kv64, &kv_full[st], (a.hq + kvh) * D + 64 * c, kv_row,
                      a.err);
          tma_load_2d(sv + st * L::kKV + c * kKs * 128, &tm_kv64, &kv_full[st], (a.hq + a.hkv + kvh) * D + 64 * c,
                      kv_row, a.err);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16_f32(kBlk, kKs, 0, 0);
      constexpr uint32_t id_dq = idesc_bf16_f32(kBlk, D, 0, 1);
      bool ok = mbar_wait(qo_tmem, 0, a.err, kErrMmaWait);  // Q, dO landed and copied into TMEM
      for (int j = 0; j <= nkv && ok; ++j) {
        if (j < nkv) {
          const int st = j % ST;
          const int s = j & 1;
          if (!mbar_wait(&kv_full[st], (j / ST) & 1, a.err, kErrMmaWait)) { ok = false; break; }
          if (!mbar_wait(&s_empty[s], ((j >> 1) & 1) ^ 1, a.err, kErrMmaWait)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sk + st * L::kKV), v_addr = smem_u32(sv + st * L::kKV);
          #pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t okv = (kk >> 2) * kKs * 128 + (kk & 3) * 32;
            umma_bf16_ts(tmem + s * kKs, t_q + kk * 8, smem_desc_sw128(k_addr + okv, 16, 1024), id_s, kk > 0);
            umma_bf16_ts(tmem + 128 + s * kKs, t_do + kk * 8, smem_desc_sw128(v_addr + okv, 16, 1024), id_s,
                         kk > 0);
          }
          umma_commit(&s_full[s]);
        }
        if (j >= 1) {
          const int p = j - 1;
          const int sp = p & 1;
          const int stp = p % ST;
          if (!mbar_wait(&ds_full[sp], (p >> 1) & 1, a.err, kErrMmaWait)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sk + stp * L::kKV);
          #pragma unroll
          for (int kk = 0; kk < kKs / 16; ++kk)  // A = dS from TMEM (packed bf16, see below)
            umma_bf16_ts(t_dq, tmem + uint32_t(sp * kKs + (kk >> 1) * 32 + (kk & 1) * 8),
                         smem_desc_sw128(k_addr + kk * 2048, kKs * 128, 1024), id_dq, (p > 0 || kk > 0));
          umma_commit(&kv_empty[stp]);
        }
      }
      if (ok) umma_commit(dq_done);
    }
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;                 // q row within the tile
    const int q_pos = qblk * kBlk + r;
    const uint32_t lane_off = uint32_t(quad * 32) << 16;
    const float sl2 = a.scale * kLog2e;
    const int64_t stat = (int64_t(b) * a.hq + h) * a.seq + q_pos;
    const float lse2 = a.lse[stat] * kLog2e;
    const float dlt = a.delta[stat];
    bool ok = mbar_wait(q_full, 0, a.err, kErrEpiWait);
    if (ok) {
      // this warp's half of its rows of Q and dO, from the swizzled tiles into TMEM
      sw128_row_to_tmem(sq, kBlk, half, r, t_q + lane_off + half * 32);
      sw128_row_to_tmem(sdo, kBlk, half, r, t_do + lane_off + half * 32);
      tmem_wait_st();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(qo_tmem);
    for (int j = 0; j < nkv; ++j) {
      const int s = j & 1;
      const uint32_t n = (j >> 1) & 1;
      const bool diag = j >= 2 * qblk;              // the sub-block reaches the q block's rows
      const int k_pos0 = j * kKs + half * 32;
      if (!mbar_wait(&s_full[s], n, a.err, kErrEpiWait)) { ok = false; break; }
      tc_fence_after();
      uint32_t s32[32], p32[32];
      tmem_ld32(tmem + s * kKs + lane_off + half * 32, s32);
      tmem_ld32(tmem + 128 + s * kKs + lane_off + half * 32, p32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[s]);
      uint32_t pk[16];
      #pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float ds[2];
        #pragma unroll
        for (int z = 0; z < 2; ++z) {
          float pv = fast_exp2(fmaf(__uint_as_float(s32[e + z]), sl2, -lse2));
          if (diag && k_pos0 + e + z > q_pos) pv = 0.f;
          ds[z] = pv * (__uint_as_float(p32[e + z]) - dlt);
        }
        pk[e / 2] = pack_bf16(ds[0], ds[1]);
      }
      // dS back into this sub-block's S TMEM buffer (the first 16 columns of this warp's
      // 32), the A operand of the dQ MMA; buffer reuse is ordered by the MMA issue order
      // as in the dK / dV kernel
      tmem_st16(tmem + s * kKs + lane_off + half * 32, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[s]);
    }
    if (ok && mbar_wait(dq_done, 0, a.err, kErrEpiWait)) {
      tc_fence_after();
      __nv_bfloat16* dst = a.out + int64_t(row0 + r) * a.out_ld + int64_t(h) * D;
      #pragma unroll 1
      for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 32) {
        uint32_t v[32];
        tmem_ld32(t_dq + lane_off + c, v);
        tmem_wait_ld();
        #pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 o;
          o.x = pack_bf16(__uint_as_float(v[8 * u + 0]) * a.scale, __uint_as_float(v[8 * u + 1]) * a.scale);
          o.y = pack_bf16(__uint_as_float(v[8 * u + 2]) * a.scale, __uint_as_float(v[8 * u + 3]) * a.scale);
          o.z = pack_bf16(__uint_as_float(v[8 * u + 4]) * a.scale, __uint_as_float(v[8 * u + 5]) * a.scale);
          o.w = pack_bf16(__uint_as_float(v[8 * u + 6]) * a.scale, __uint_as_float(v[8 * u + 7]) * a.scale);
          *reinterpret_cast<uint4*>(dst + c + 8 * u) = o;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <class K>
void set_smem(K kernel, int bytes) {
  RESIHP_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

void check_shapes(int rows, int seq, int hq, int hkv, int d) {
  RESIHP_CHECK(d == 64 || d == 128, "attention head_dim must be 64 or 128, got ", d);
  RESIHP_CHECK(seq % kBlk == 0 && rows % seq == 0, "attention needs seq % 128 == 0 and rows % seq == 0");
  RESIHP_CHECK(hkv > 0 && hq % hkv == 0, "query heads must be a multiple of kv heads");
}

}  // namespace

void attn_fwd(const void* qkv, int64_t qkv_ld, void* out, int64_t out_ld, float* lse, int rows, int seq, int hq,
              int hkv, int d, float scale, int* err, cudaStream_t st) {
  check_shapes(rows, seq, hq, hkv, d);
  const CUtensorMap tm = make_tma_2d_bf16(qkv, rows, int64_t(hq + 2 * hkv) * d, qkv_ld, 64, kBlk);
  AttnArgs a{static_cast<__nv_bfloat16*>(out), lse, nullptr, nullptr, seq, hq, hkv, d, out_ld, 0, scale, err};
  dim3 grid(hq, rows / seq, seq / kBlk);
  if (d == 128) {
    set_smem(attn_fwd_kernel<128>, FwdSmem<128>::kBytes);
    launch_pdl(attn_fwd_kernel<128>, grid, kFwdThreads, FwdSmem<128>::kBytes, st, tm, a);
  } else {
    set_smem(attn_fwd_kernel<64>, FwdSmem<64>::kBytes);
    launch_pdl(attn_fwd_kernel<64>, grid, kFwdThreads, FwdSmem<64>::kBytes, st, tm, a);
  }
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

void attn_bwd(const void* qkv, int64_t qkv_ld, const void* out, int64_t out_ld, const void* dout, int64_t dout_ld,
              const float* lse, float* delta, void* dqkv, int64_t dqkv_ld, int rows, int seq, int hq, int hkv, int d,
              float scale, int* err, cudaStream_t st) {
  check_shapes(rows, seq, hq, hkv, d);
  RESIHP_CHECK(dqkv_ld == int64_t(hq + 2 * hkv) * d, "dqkv must be dense");
  {
    const int warps = rows * hq;
    launch_pdl(attn_delta_kernel, ((warps + 3) / 4 * 32 + 255) / 256, 256, 0, st, static_cast<const __nv_bfloat16*>(out), out_ld,
                                                                static_cast<const __nv_bfloat16*>(dout), dout_ld,
                                                                delta, rows, seq, hq, d);
    RESIHP_CUDA_CHECK(cudaGetLastError());
  }
  const CUtensorMap tm = make_tma_2d_bf16(qkv, rows, int64_t(hq + 2 * hkv) * d, qkv_ld, 64, kBlk);
  const CUtensorMap tm_do = make_tma_2d_bf16(dout, rows, int64_t(hq) * d, dout_ld, 64, kBlk);
  const CUtensorMap tm_q64 = make_tma_2d_bf16(qkv, rows, int64_t(hq + 2 * hkv) * d, qkv_ld, 64, kQs);  // also K, V rows
  const CUtensorMap tm_do64 = make_tma_2d_bf16(dout, rows, int64_t(hq) * d, dout_ld, 64, kQs);
  RESIHP_CHECK(reinterpret_cast<uintptr_t>(lse) % 16 == 0 && reinterpret_cast<uintptr_t>(delta) % 16 == 0,
               "attention statistics must be 16-byte aligned");
  AttnArgs a{static_cast<__nv_bfloat16*>(dqkv), const_cast<float*>(lse), static_cast<const __nv_bfloat16*>(dout),
             delta, seq, hq, hkv, d, dqkv_ld, dout_ld, scale, err};
  dim3 grid_kv(hkv, rows / seq, seq / kBlk);
  dim3 grid_q(hq, rows / seq, seq / kBlk);
  if (d == 128) {
    set_smem(attn_bwd_dkdv_kernel<128>, DkdvSmem<128>::kBytes);
    launch_pdl(attn_bwd_dkdv_kernel<128>, grid_kv, kDkdvThreads, DkdvSmem<128>::kBytes, st, tm, tm_q64, tm_do64, a);
    RESIHP_CUDA_CHECK(cudaGetLastError());
    set_smem(attn_bwd_dq_kernel<128>, DqSmem<128>::kBytes);
    launch_pdl(attn_bwd_dq_kernel<128>, grid_q, kDkdvThreads, DqSmem<128>::kBytes, st, tm, tm_do, tm_q64, a);
  } else {
    set_smem(attn_bwd_dkdv_kernel<64>, DkdvSmem<64>::kBytes);
    launch_pdl(attn_bwd_dkdv_kernel<64>, grid_kv, kDkdvThreads, DkdvSmem<64>::kBytes, st, tm, tm_q64, tm_do64, a);
    RESIHP_CUDA_CHECK(cudaGetLastError());
    set_smem(attn_bwd_dq_kernel<64>, DqSmem<64>::kBytes);
    launch_pdl(attn_bwd_dq_kernel<64>, grid_q, kDkdvThreads, DqSmem<64>::kBytes, st, tm, tm_do, tm_q64, a);
  }
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

}  // namespace resihp
