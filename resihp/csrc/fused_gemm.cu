// Tensor-parallel GEMMs fused with their sequence-parallel collective over NVLink peer
// memory (CUDA IPC mappings of each rank's symmetric workspace; plain P2P loads and
// stores plus flag words -- no multicast of any kind). Reference counterparts: the
// column/row-parallel ``F.linear`` calls with the Megatron ``f`` / ``g`` all-reduces
// (resihp/parallel/tp.py:63-89, 235-249); here with sequence parallelism the pair
// becomes all-gather / reduce-scatter over tokens, fused into the GEMM.
//
//   AG->GEMM   y[T, N]      = all_gather_tokens(x_r[T/tp, K]) * op(W)
//   GEMM->RS   y_r[T/tp, N] = reduce_scatter_tokens(h[T, K] * op(W))
//
// Both are the persistent tcgen05 GEMM of gemm.cu (TMA producer warp, one MMA-issuing
// thread, four epilogue warps, two TMEM accumulators) plus *copy warps* (four or six per
// CTA, see CopyCfg) that move the collective's data with coalesced 16-byte loads and
// stores while the tensor cores work; every remote byte crosses NVLink exactly once.
//
// AG: the copy warps first publish this rank's chunk -- one pass writes it into the
// rank's symmetric slot (epoch parity) and into the local gather buffer -- and the last
// copy warp to finish flags the epoch to every peer. They then pull their CTA's share of
// each peer's slot into the gather buffer and bump that chunk's ready counter. Tiles run
// own chunk first (read in place through this rank's tensor map), then the peers' chunks
// once their counters are complete. The gather buffer ends up holding the whole gathered
// input, reused by the backward pass for the weight gradient.
//
// RS: tiles of the peers' token chunks run first; their epilogue writes the partial tile
// to this rank's own partial buffer (epoch parity) and bumps that tile's flag. Each CTA's
// copy warps pull, for every own-chunk tile that CTA will finish, the peers' partial tiles
// once flagged, into a local receive buffer; the own tile's epilogue then sums all ranks'
// partials in rank order (fp32, deterministic) and writes the reduced rows.
//
// Buffer reuse needs no extra handshake: a rank reaches epoch e only after its epoch e-1
// kernel consumed every peer's epoch e-1 data, which those peers produced only after
// finishing their epoch e-2 kernels -- the last readers of this parity's buffers.
//
// Every wait (peer flags, counters, mbarriers) is bounded by the global timer and reports
// into the error word. All CTAs must be resident together (grid <= SM count, one CTA
// per SM); if that ever failed, the bounded waits would turn it into an error, not a hang.
#include <algorithm>
#include <cstring>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "launch.h"

namespace resihp {

constexpr int kMaxTp = 8;

// Copy-warp configuration per kernel variant.
//   V = 0: four copy warps, eight 16-byte loads in flight per thread; the AG pull gives
//          every CTA a slice of every peer chunk and a chunk's tiles start once all CTAs
//          finished it (validated at TP2).
//   V = 1: six copy warps, sixteen loads in flight per thread; the AG pull hands out
//          (peer chunk, row block, row slice) units and a tile starts as soon as its own
//          128-row block is complete; the RS pull gives each copy warp a fixed subset of
//          the peers and takes whichever of them is ready first (for TP > 2).
template <int V>
struct CopyCfg {
  static constexpr int kWarps = V == 0 ? 4 : 6;
  static constexpr int kUnroll = V == 0 ? 8 : 16;
  static constexpr int kThreads = 192 + 32 * kWarps;
};

struct CommArgs {
  int rank, tp, rows_per_rank;
  unsigned epoch;
  // AG
  const __nv_bfloat16* peer_slot[kMaxTp];  // each rank's slot for this epoch
  __nv_bfloat16* own_slot;                 // this rank's slot for this epoch
  __nv_bfloat16* xg;                       // local gather buffer [T, K]
  const __nv_bfloat16* x_local;            // this rank's chunk [T/tp, K]
  int64_t ldx;
  unsigned* sig_ag;                        // local: sig_ag[s] = last epoch rank s published
  unsigned* peer_sig_ag[kMaxTp];           // each rank's sig_ag array
  unsigned* pub;                           // local publish counter
  unsigned pub_target;
  unsigned* ready;                         // local per-chunk ready counters [tp] (V = 0)
  unsigned ready_target;
  unsigned* rb_ready;                      // local per-row-block ready counters [tp * T/tp/128] (V = 1)
  unsigned rb_target;
  int slices;                              // row slices per 128-row block in the V = 1 pull
  // RS
  __nv_bfloat16* part_local;               // this rank's partial buffer [T, N] for this epoch
  const __nv_bfloat16* peer_part[kMaxTp];  // each rank's partial buffer for this epoch
  unsigned* flag_local;                    // this rank's per-tile flags
  const unsigned* peer_flag[kMaxTp];       // each rank's per-tile flags
  unsigned flag_target;
  __nv_bfloat16* recv;                     // local receive buffer [tp][T/tp, N]
};

struct FusedArgs {
  void* c;  // AG: y [T, N]; RS: y_r [T/tp, N]
  int64_t ldc;
  int m, n, k;
  int* err;
  uint64_t wait_ns;  // budget of each wait on a peer's flag or a pull counter
  CommArgs comm;
};

// One lane waits, the whole warp learns the outcome.
__device__ __forceinline__ bool warp_wait_geq(const unsigned* p, unsigned target, int* err, int lane,
                                              uint64_t budget_ns) {
  int ok = 1;
  if (lane == 0) ok = wait_geq(p, target, err, kErrPeerWait, budget_ns) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Copy `rows` rows of `cols16` 16-byte vectors (row strides in vectors) with `kT` threads
// (thread index `ct`), `kU` loads in flight per thread.
template <int kT, int kU>
__device__ __forceinline__ void copy_rows(uint4* dst, int64_t dld, const uint4* src, int64_t sld, int rows,
                                          int cols16, int ct, int* err) {
  // checked build: both ends of a 16-byte vector copy on 16-byte boundaries, rows no
  // wider than their strides
  if (!bounds_ok(((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u) == 0 &&
                     cols16 <= dld && cols16 <= sld,
                 err))
    return;
  const int64_t total = int64_t(rows) * cols16;
  for (int64_t base = ct; base < total; base += int64_t(kT) * kU) {
    uint4 r[kU];
    #pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + int64_t(u) * kT;
      if (i < total) r[u] = ld_cg_v4(src + (i / cols16) * sld + (i % cols16));
    }
    #pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + int64_t(u) * kT;
      if (i < total) dst[(i / cols16) * dld + (i % cols16)] = r[u];
    }
  }
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
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 512;
};

// Tile t -> (chunk, m0, tn). Chunks are visited starting at (rank + first) % tp; inside a
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
  m0 = chunk * c.rows_per_rank + (g0 + in_group % size) * kFBM;
  tn_out = in_group / size;
}

template <int BN, bool B_MN, int MODE, int V>
__global__ void __launch_bounds__(CopyCfg<V>::kThreads, 1)
    fused_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_a2,
                      const __grid_constant__ CUtensorMap tma_b, FusedArgs g) {
  using S = FusedShape<BN>;
  constexpr int kCW = CopyCfg<V>::kWarps;
  constexpr int kCT = 32 * kCW;
  constexpr int kCU = CopyCfg<V>::kUnroll;
  constexpr int kStages = S::kStages;
  constexpr int kPullSlots = 4;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * S::kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* pulled = acc_empty + 2;  // RS: own tile j's peer partials are in `recv`
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pulled + kPullSlots);

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
    for (int j = 0; j < kPullSlots; ++j) mbar_init(&pulled[j], kCW);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch(&tma_a);
      tma_prefetch(&tma_b);
      if (MODE == 1) tma_prefetch(&tma_a2);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int ready_key = -1;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int chunk, m0, tn;
        fused_tile(t, tiles_m_chunk, tiles_n, cm, first, chunk, m0, tn);
        const int n0 = tn * BN;
        const bool own = chunk == cm.rank;
        if (MODE == 1 && !own) {
          // V = 0: the whole peer chunk; V = 1: only this tile's 128-row block
          const int key = V == 0 ? chunk : chunk * tiles_m_chunk + (m0 - chunk * cm.rows_per_rank) / kFBM;
          if (key != ready_key) {
            const bool arrived = V == 0 ? wait_geq(cm.ready + key, cm.ready_target, g.err, kErrPeerWait, g.wait_ns)
                                        : wait_geq(cm.rb_ready + key, cm.rb_target, g.err, kErrPeerWait, g.wait_ns);
            if (!arrived) { ok = false; break; }
            fence_proxy_async_global();
            ready_key = key;
          }
        }
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, g.err, kErrTmaWait)) { ok = false; break; }
          uint8_t* sa = smem + s * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_expect_tx(&full[s], S::kStageBytes);
          const int k0 = kb * kFBK;
          if (MODE == 1 && own) tma_load_2d(sa, &tma_a, &full[s], k0, m0 - cm.rank * cm.rows_per_rank, g.err);
          else if (MODE == 1) tma_load_2d(sa, &tma_a2, &full[s], k0, m0, g.err);
          else tma_load_2d(sa, &tma_a, &full[s], k0, m0, g.err);
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
    // ---------------- MMA issuer ----------------
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
        if (!tmem_span_ok(d, tmem_base, 2 * BN, BN, g.err)) break;
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
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    int i = 0;
    int j_own = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
      int chunk, m0, tn;
      fused_tile(t, tiles_m_chunk, tiles_n, cm, first, chunk, m0, tn);
      const int a = i & 1;
      const uint32_t accph = (i >> 1) & 1;
      if (!mbar_wait(&acc_full[a], accph, g.err, kErrEpiWait)) break;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const int lrow = row - chunk * cm.rows_per_rank;
      const bool reduce_here = MODE == 2 && chunk == cm.rank;
      __nv_bfloat16* dst;
      if (MODE == 1) dst = static_cast<__nv_bfloat16*>(g.c) + int64_t(row) * g.ldc;
      else if (!reduce_here) dst = cm.part_local + int64_t(row) * g.n;
      else dst = static_cast<__nv_bfloat16*>(g.c) + int64_t(lrow) * g.ldc;
      if (reduce_here) {
        const int slot = j_own % kPullSlots;
        if (!mbar_wait(&pulled[slot], (j_own / kPullSlots) & 1, g.err, kErrEpiWait)) ok = false;
        ++j_own;
      }
      #pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t v[32];
        const uint32_t ta = tmem_base + a * BN + cc * 32 + (uint32_t(q * 32) << 16);
        if (!tmem_span_ok(ta, tmem_base, 2 * BN, 32, g.err)) continue;
        tmem_ld32(ta, v);
        tmem_wait_ld();
        const int col0 = tn * BN + cc * 32;
        if (!ok || col0 >= g.n) continue;
        float f[32];
        #pragma unroll
        for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(v[e]);
        if (reduce_here) {
          // every rank's partial, summed in rank order (this rank's own in fp32)
          float tot[32];
          #pragma unroll
          for (int e = 0; e < 32; ++e) tot[e] = 0.f;
          for (int src = 0; src < cm.tp; ++src) {
            if (src == cm.rank) {
              #pragma unroll
              for (int e = 0; e < 32; ++e) tot[e] += f[e];
              continue;
            }
            const __nv_bfloat16* p = cm.recv + (int64_t(src) * cm.rows_per_rank + lrow) * g.n + col0;
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
      if (MODE == 2 && !reduce_here) {
        // flag this warp's 32 rows of the partial tile (four flags per tile, one per warp)
        __threadfence_system();
        __syncwarp();
        if (lane == 0) atomicAdd(cm.flag_local + (m0 / kFBM) * tiles_n + tn, 1u);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
  } else {
    // ---------------- copy warps ----------------
    const int ct = threadIdx.x - 192;  // 0 .. kCT-1
    bool ok = true;
    if (MODE == 1) {
      const int cols16 = int(cm.ldx / 8);
      const int lo = int(int64_t(cm.rows_per_rank) * blockIdx.x / gridDim.x);
      const int hi = int(int64_t(cm.rows_per_rank) * (blockIdx.x + 1) / gridDim.x);
      // publish: this CTA's rows of the own chunk -> own slot and gather buffer
      {
        const uint4* src = reinterpret_cast<const uint4*>(cm.x_local + int64_t(lo) * cm.ldx);
        uint4* slot = reinterpret_cast<uint4*>(cm.own_slot + int64_t(lo) * cm.ldx);
        uint4* xg = reinterpret_cast<uint4*>(cm.xg + (int64_t(cm.rank) * cm.rows_per_rank + lo) * cm.ldx);
        const int64_t total = int64_t(hi - lo) * cols16;
        for (int64_t v = ct; v < total; v += kCT) {
          const uint4 x = src[v];
          slot[v] = x;
          xg[v] = x;
        }
        __threadfence_system();
        __syncwarp();
        if (lane == 0) {
          const unsigned prev = atomicAdd(cm.pub, 1u);
          if (prev + 1 == cm.pub_target) {
            // the last copy warp of the grid announces the epoch to every peer
            __threadfence_system();
            for (int p = 0; p < cm.tp; ++p)
              if (p != cm.rank) st_release_sys(cm.peer_sig_ag[p] + cm.rank, cm.epoch);
          }
        }
      }
      if (V == 0) {
        // pull: this CTA's rows of every peer chunk
        for (int p = 1; p < cm.tp && ok; ++p) {
          const int chunk = (cm.rank + p) % cm.tp;
          ok = warp_wait_geq(cm.sig_ag + chunk, cm.epoch, g.err, lane, g.wait_ns);
          if (!ok) break;
          copy_rows<kCT, kCU>(
              reinterpret_cast<uint4*>(cm.xg + (int64_t(chunk) * cm.rows_per_rank + lo) * cm.ldx), cols16,
              reinterpret_cast<const uint4*>(cm.peer_slot[chunk] + int64_t(lo) * cm.ldx), cols16, hi - lo, cols16,
              ct, g.err);
          fence_proxy_async_global();
          __threadfence();
          __syncwarp();
          if (lane == 0) atomicAdd(cm.ready + chunk, 1u);
        }
      } else {
        // pull: units (peer chunk, 128-row block, row slice) in the order the tiles need
        // them; every copy warp bumps the block's counter after its share of a unit
        const int blocks = tiles_m_chunk;
        const int slices = cm.slices;
        const int srows = kFBM / slices;
        const int units = (cm.tp - 1) * blocks * slices;
        int announced = -1;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
          const int chunk = (cm.rank + 1 + u / (blocks * slices)) % cm.tp;
          const int rb = (u / slices) % blocks;
          const int r0 = rb * kFBM + (u % slices) * srows;
          if (chunk != announced) {
            ok = warp_wait_geq(cm.sig_ag + chunk, cm.epoch, g.err, lane, g.wait_ns);
            if (!ok) break;
            announced = chunk;
          }
          copy_rows<kCT, kCU>(
              reinterpret_cast<uint4*>(cm.xg + (int64_t(chunk) * cm.rows_per_rank + r0) * cm.ldx), cols16,
              reinterpret_cast<const uint4*>(cm.peer_slot[chunk] + int64_t(r0) * cm.ldx), cols16, srows, cols16, ct, g.err);
          fence_proxy_async_global();
          __threadfence();
          __syncwarp();
          if (lane == 0) atomicAdd(cm.rb_ready + chunk * blocks + rb, 1u);
        }
      }
    } else {
      // for each own-chunk tile this CTA will reduce: pull the peers' partial tiles
      int j = 0;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int chunk, m0, tn;
        fused_tile(t, tiles_m_chunk, tiles_n, cm, first, chunk, m0, tn);
        if (chunk != cm.rank) continue;
        const int lrow0 = m0 - chunk * cm.rows_per_rank;
        const int ncols16 = min(BN, g.n - tn * BN) / 8;
        const int flag = (m0 / kFBM) * tiles_n + tn;
        if (V == 0) {
          for (int src = 0; src < cm.tp && ok; ++src) {
            if (src == cm.rank) continue;
            ok = warp_wait_geq(cm.peer_flag[src] + flag, cm.flag_target, g.err, lane, g.wait_ns);
            if (!ok) break;
            const uint4* from = reinterpret_cast<const uint4*>(cm.peer_part[src] + int64_t(m0) * g.n + tn * BN);
            uint4* to = reinterpret_cast<uint4*>(cm.recv + (int64_t(src) * cm.rows_per_rank + lrow0) * g.n + tn * BN);
            copy_rows<kCT, kCU>(to, g.n / 8, from, g.n / 8, kFBM, ncols16, ct, g.err);
          }
        } else {
          // this warp's peers (every kCW-th peer), copied in the order their tiles arrive
          const int cw = ct >> 5;
          unsigned pending = 0;
          for (int src = 0, i = 0; src < cm.tp; ++src) {
            if (src == cm.rank) continue;
            if (i++ % kCW == cw) pending |= 1u << src;
          }
          const uint64_t start = globaltimer();
          while (pending != 0 && ok) {
            int got = -1;
            if (lane == 0) {
              for (int src = 0; src < cm.tp && got < 0; ++src)
                if ((pending >> src & 1u) && static_cast<int>(ld_acquire_sys(cm.peer_flag[src] + flag) - cm.flag_target) >= 0)
                  got = src;
              if (got < 0 && globaltimer() - start > g.wait_ns) {
                record_error(g.err, kErrPeerWait);
                got = -2;
              }
            }
            got = __shfl_sync(0xffffffffu, got, 0);
            if (got == -2) { ok = false; break; }
            if (got < 0) continue;
            const uint4* from = reinterpret_cast<const uint4*>(cm.peer_part[got] + int64_t(m0) * g.n + tn * BN);
            uint4* to = reinterpret_cast<uint4*>(cm.recv + (int64_t(got) * cm.rows_per_rank + lrow0) * g.n + tn * BN);
            copy_rows<32, kCU>(to, g.n / 8, from, g.n / 8, kFBM, ncols16, lane, g.err);
            pending &= ~(1u << got);
          }
        }
        __threadfence_block();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pulled[j % kPullSlots]);
        ++j;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
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

template <int BN, bool B_MN, int MODE, int V>
void launch_fused_v(const CUtensorMap& ta, const CUtensorMap& ta2, const CUtensorMap& tb, FusedArgs g, int grid,
                    cudaStream_t st) {
  using S = FusedShape<BN>;
  auto kernel = fused_gemm_kernel<BN, B_MN, MODE, V>;
  RESIHP_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem));
  // The grid never exceeds the SM count and one CTA fills an SM, so on a GPU this process
  // owns every CTA is resident at once.
  kernel<<<grid, CopyCfg<V>::kThreads, S::kSmem, st>>>(ta, ta2, tb, g);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

template <int BN, bool B_MN, int MODE>
void launch_fused(const CUtensorMap& ta, const CUtensorMap& ta2, const CUtensorMap& tb, FusedArgs g, int grid,
                  int variant, cudaStream_t st) {
  if (variant == 0) launch_fused_v<BN, B_MN, MODE, 0>(ta, ta2, tb, g, grid, st);
  else launch_fused_v<BN, B_MN, MODE, 1>(ta, ta2, tb, g, grid, st);
}

int copy_warps(int variant) { return variant == 0 ? CopyCfg<0>::kWarps : CopyCfg<1>::kWarps; }

// Row slices per 128-row block in the V = 1 AG pull: enough units for every CTA.
int ag_slices(int rows_per_rank, int tp, int grid) {
  const int units = (tp - 1) * (rows_per_rank / kFBM);
  int s = 1;
  while (s < 16 && units * s < grid) s *= 2;
  return s;
}

}  // namespace

// Per launch, every copy warp of the grid bumps the AG publish counter once and (V = 0)
// each chunk's ready counter once; the host advances its bases by this much per call.
int fused_counter_step(int grid, int variant) { return copy_warps(variant) * grid; }

// Per launch (V = 1), every peer 128-row block's ready counter grows by this much.
int fused_block_step(int t_rows, int n, int tp, int grid) {
  return ag_slices(t_rows / tp, tp, grid) * copy_warps(1);
}

int fused_grid(int m, int n, int tp) {
  (void)tp;
  const int tiles = (m / kFBM) * ((n + 255) / 256);
  return std::min(tiles, sm_count());
}

void ag_gemm(const void* x_local, void* own_slot, const void* const* peer_slot, void* xg, const void* w,
             int64_t ldw, bool w_mn, void* y, int64_t ldy, int t_rows, int n, int k, int rank, int tp,
             unsigned epoch, unsigned* sig_ag, unsigned* const* peer_sig_ag, unsigned* pub, unsigned pub_base,
             unsigned* ready, unsigned ready_base, unsigned* rb_ready, unsigned rb_base, int variant, int grid,
             int* err, cudaStream_t st) {
  RESIHP_CHECK(tp >= 2 && tp <= kMaxTp && t_rows % tp == 0 && (t_rows / tp) % kFBM == 0,
               "ag_gemm: rows per rank must be a multiple of 128");
  RESIHP_CHECK(variant == 0 || (variant == 1 && rb_ready != nullptr), "ag_gemm: unknown variant");
  RESIHP_CHECK(n % 8 == 0 && k % 8 == 0, "ag_gemm: N and K must be multiples of 8");
  const int tl = t_rows / tp;
  CUtensorMap ta = make_tma_2d_bf16(x_local, tl, k, k, 64, kFBM);
  CUtensorMap ta2 = make_tma_2d_bf16(xg, t_rows, k, k, 64, kFBM);
  CUtensorMap tb = w_mn ? make_tma_2d_bf16(w, k, n, ldw, 64, 64) : make_tma_2d_bf16(w, n, k, ldw, 64, 256);
  FusedArgs g{};
  g.c = y;
  g.ldc = ldy;
  g.m = t_rows;
  g.n = n;
  g.k = k;
  g.err = err;
  g.wait_ns = peer_wait_budget_ns();
  CommArgs& c = g.comm;
  c.rank = rank;
  c.tp = tp;
  c.rows_per_rank = tl;
  c.epoch = epoch;
  for (int p = 0; p < tp; ++p) {
    c.peer_slot[p] = static_cast<const __nv_bfloat16*>(peer_slot[p]);
    c.peer_sig_ag[p] = peer_sig_ag[p];
  }
  c.own_slot = static_cast<__nv_bfloat16*>(own_slot);
  c.xg = static_cast<__nv_bfloat16*>(xg);
  c.x_local = static_cast<const __nv_bfloat16*>(x_local);
  c.ldx = k;
  c.sig_ag = sig_ag;
  c.pub = pub;
  c.pub_target = pub_base + unsigned(fused_counter_step(grid, variant));
  c.ready = ready;
  c.ready_target = ready_base + unsigned(fused_counter_step(grid, variant));
  c.rb_ready = rb_ready;
  c.slices = ag_slices(tl, tp, grid);
  c.rb_target = rb_base + unsigned(variant == 1 ? fused_block_step(t_rows, n, tp, grid) : 0);
  if (w_mn) launch_fused<256, true, 1>(ta, ta2, tb, g, grid, variant, st);
  else launch_fused<256, false, 1>(ta, ta2, tb, g, grid, variant, st);
}

void gemm_rs(const void* h, const void* w, int64_t ldw, bool w_mn, void* y_local, int64_t ldy, int t_rows, int n,
             int k, int rank, int tp, unsigned epoch, void* part_local, const void* const* peer_part,
             unsigned* flag_local, const unsigned* const* peer_flag, void* recv, int variant, int grid, int* err,
             cudaStream_t st) {
  RESIHP_CHECK(tp >= 2 && tp <= kMaxTp && t_rows % tp == 0 && (t_rows / tp) % kFBM == 0,
               "gemm_rs: rows per rank must be a multiple of 128");
  RESIHP_CHECK(variant == 0 || variant == 1, "gemm_rs: unknown variant");
  RESIHP_CHECK(n % 32 == 0 && k % 8 == 0, "gemm_rs: N must be a multiple of 32 and K of 8");
  const int tl = t_rows / tp;
  CUtensorMap ta = make_tma_2d_bf16(h, t_rows, k, k, 64, kFBM);
  CUtensorMap tb = w_mn ? make_tma_2d_bf16(w, k, n, ldw, 64, 64) : make_tma_2d_bf16(w, n, k, ldw, 64, 256);
  FusedArgs g{};
  g.c = y_local;
  g.ldc = ldy;
  g.m = t_rows;
  g.n = n;
  g.k = k;
  g.err = err;
  g.wait_ns = peer_wait_budget_ns();
  CommArgs& c = g.comm;
  c.rank = rank;
  c.tp = tp;
  c.rows_per_rank = tl;
  c.epoch = epoch;
  c.part_local = static_cast<__nv_bfloat16*>(part_local);
  for (int p = 0; p < tp; ++p) {
    c.peer_part[p] = static_cast<const __nv_bfloat16*>(peer_part[p]);
    c.peer_flag[p] = peer_flag[p];
  }
  c.flag_local = flag_local;
  c.flag_target = 4u * epoch;  // four warp flags per tile per call
  c.recv = static_cast<__nv_bfloat16*>(recv);
  if (w_mn) launch_fused<256, true, 2>(ta, ta, tb, g, grid, variant, st);
  else launch_fused<256, false, 2>(ta, ta, tb, g, grid, variant, st);
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
