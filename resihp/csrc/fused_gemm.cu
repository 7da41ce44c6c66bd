// Tensor-parallel GEMMs fused with their collective over NVLink peer memory (CUDA IPC
// mappings of each rank's symmetric workspace; posted P2P stores, P2P reductions on
// counter words and TMA loads of this GPU's own memory -- no multicast of any kind).
// Reference counterparts: the column/row-parallel ``F.linear`` calls with the Megatron
// ``f`` / ``g`` all-reduces (resihp/parallel/tp.py:63-89, 235-249). With sequence
// parallelism the pair becomes all-gather / reduce-scatter over tokens; without it the
// row-parallel output (and the column-parallel input gradient) is an all-reduce.
//
//   AG->GEMM   y[T, N]      = all_gather_tokens(x_r[T/tp, K]) * op(W)
//   GEMM->RS   y_r[T/tp, N] = reduce_scatter_tokens(h[T, K] * op(W))
//   GEMM->AR   y[T, N]      = all_reduce(h[T, K] * op(W))
//
// All three are the persistent tcgen05 GEMM of gemm.cu (TMA producer warp, one
// MMA-issuing thread, four epilogue warps, two TMEM accumulators) plus four copy warps.
// Data moves by *push*: the rank that owns a piece of data stores it straight into the
// peer's workspace (posted NVLink writes, no round trip per load) and then adds to a
// counter word in the peer's memory with a release reduction; the consumer acquires the
// counter and reads its own memory.
//
// AG: the copy warps push this rank's chunk, in units of a few rows, into every peer's
//     landing zone, destination-major in the order the peers consume it (peer r-1
//     first: it computes chunk r right after its own), and count each 128-row block per
//     (source, block). Pushes are bulk asynchronous copies driven by one thread (TMA
//     engine: global -> shared staging -> peer global, two 16 KB buffers), so the bytes
//     in flight do not cost registers. The producer loads own-chunk tiles from x_local and a peer chunk's
//     tiles from the local landing zone once that block's counter is complete. The copy
//     warps then also assemble the gathered input in ``xg`` for the backward pass.
// RS: tiles of the peers' token chunks run first; their epilogue stores the bf16 partial
//     in a local, tile-contiguous send buffer and flags it, and the copy warps push each
//     finished 64 KB tile as one bulk copy into the owning peer's (tile-contiguous)
//     receive buffer and count it there.
//     Own-chunk tiles run last: their epilogue stores this rank's partial in y, and once
//     the tp-1 contributions have arrived the copy warps add them, many rows in flight.
//     The peers' partials travel as bf16 (as in a bf16 reduce-scatter); the sum is taken
//     in fp32 in a fixed order (own partial first, then the peers' in rank order), so it
//     is deterministic.
//     (The tile counters come in two banks by call parity: a fast source may already be
//     contributing to the next call.)
// AR: RS, where the copy warps also stage each reduced slice of an own tile and bulk-push
//     it into every peer's (tile-contiguous) output landing zone and count it there, then
//     copy the other owners' tiles from there into y.
//
// Work is claimed dynamically -- output tiles by the producer, copy items by the copy
// warps -- from per-call counters in the same global order on every rank (peer data
// before data that waits on peers), so no CTA ever waits for another CTA of its own
// grid: the kernels need no co-residency of their CTAs, only that each rank's kernel
// runs at all. Every wait (peer counters, mbarriers) is bounded by the global timer
// and reports into the error word.
//
// Buffer reuse needs no extra handshake: landing zones and receive buffers alternate
// by call parity; a rank writes a peer's parity-p buffer in call e only after finishing
// call e-1, which needed data the peer produced in its call e-1 -- after it had
// finished call e-2, the last reader of that parity. (No counterpart in the reference.)
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "launch.h"

namespace resihp {

namespace {

constexpr int kFBM = 128;
constexpr int kFBK = 64;
constexpr int kCopyWarps = 4;
constexpr int kCopyThreads = 32 * kCopyWarps;
constexpr int kFusedThreads = 192 + kCopyThreads;
constexpr int kTileRing = 4;
constexpr int kCopyUnroll = 8;  // 16-byte vectors in flight per thread in copy_rows
constexpr int kSpanUnroll = 16; // ... in copy_span (AG pushes: more bytes in flight per SM over NVLink)
constexpr int kCopyBatch = 8;   // most AG copy items per claim
constexpr int kChunk = 16384;   // bytes per bulk-push chunk (two shared-memory buffers of it)

// AG copy items per claim: up to kCopyBatch (fewer claims and system fences), but small
// enough that the items spread over every CTA's copy warps -- a push's rate over NVLink
// is set by the bytes each SM keeps in flight, so concentrating the pushes on a few CTAs
// would starve the link.
__host__ __device__ inline int ag_copy_batch(int items, int grid) {
  const int b = items / (2 * grid);
  return b < 1 ? 1 : (b > kCopyBatch ? kCopyBatch : b);
}
// An own tile's reduction is split into this many copy items (row slices): enough items
// to give every CTA's copy warps one (at least 1, at most 8 slices of 16 rows).
__host__ __device__ inline int red_slices(int per_chunk, int grid) {
  int s = 1;
  while (s < 8 && per_chunk * s < grid) s *= 2;
  return s;
}

enum FusedMode : int { kModeAG = 1, kModeRS = 2, kModeAR = 3 };

struct FusedArgs {
  void* c;  // AG, AR: y [T, N]; RS: y_r [T/tp, N]
  int64_t ldc;
  int m, n, k;
  int* err;
  uint64_t wait_ns;  // budget of each wait on a peer's counter
  const __nv_bfloat16* x_local;  // AG: this rank's chunk [T/tp, K], row stride K
  __nv_bfloat16* xg;             // AG: gathered copy [T, K] for the backward (nullptr: none)
  uint64_t* trace;               // profiling aid: [grid][kTraceSlots] timer stamps, or null
  int push_depth;                // RS / AR partial-tile pushes a copy thread keeps in flight (1 or 2)
  FusedPeers p;
};

// Profiling aid (off unless a trace buffer is set with set_fused_trace): every CTA
// records global-timer stamps at fixed points: 0 start, 1 producer done claiming,
// 2-9 epilogue end of its first 8 tiles, 10-25 (start, end) of its first 8 copy claims,
// 26-33 the claimed item of each, 34 end.
constexpr int kTraceSlots = 40;
#define FUSED_STAMP(slot, value)                                              \
  do {                                                                        \
    if (g.trace != nullptr) g.trace[blockIdx.x * kTraceSlots + (slot)] = (value); \
  } while (0)

template <int BN>
struct FusedShape {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = kFBM * kFBK * 2;
  static constexpr int kBBytes = BN * kFBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kSmem = kStages * kStageBytes + 2 * kChunk + 1024 + 512;
  static constexpr int kTileElems = kFBM * BN;  // one tile in the RS send / receive buffers
};

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void copy_bar() { asm volatile("bar.sync 1, %0;" ::"r"(kCopyThreads) : "memory"); }

__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Eight bf16 (a 16-byte vector, low half first) to fp32, exactly, without taking the
// vector's address (which would keep a register array in local memory).
__device__ __forceinline__ void bf16x8_to_f32(const uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  #pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// arr[i] by a select over every slot: a runtime index into a kernel-parameter array
// would make the compiler copy the array to local memory.
template <class T>
__device__ __forceinline__ T pick(const T (&arr)[kFusedMaxTp], int i) {
  T r = arr[0];
  #pragma unroll
  for (int q = 1; q < kFusedMaxTp; ++q)
    if (q == i) r = arr[q];
  return r;
}

// ``count`` contiguous 16-byte vectors, copy-warp thread ``ct`` of kCopyThreads,
// kSpanUnroll loads in flight per thread before their stores.
__device__ __forceinline__ void copy_span(uint4* dst, const uint4* src, int64_t count, int ct, int* err) {
  if (!bounds_ok(((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u) == 0, err)) return;
  for (int64_t base = ct; base < count; base += int64_t(kCopyThreads) * kSpanUnroll) {
    uint4 r[kSpanUnroll];
    #pragma unroll
    for (int u = 0; u < kSpanUnroll; ++u) {
      const int64_t i = base + int64_t(u) * kCopyThreads;
      if (i < count) r[u] = ld_cg_v4(src + i);
    }
    #pragma unroll
    for (int u = 0; u < kSpanUnroll; ++u) {
      const int64_t i = base + int64_t(u) * kCopyThreads;
      if (i < count) dst[i] = r[u];
    }
  }
}

// ``rows`` rows of ``cols16`` (at most 32) 16-byte vectors with their own row strides (in
// vectors): one warp per row, each lane one vector, kCopyUnroll rows in flight per warp
// before their stores (a 256-column bf16 tile row is one 512-byte warp access).
__device__ __forceinline__ void copy_rows(uint4* dst, int64_t dld, const uint4* src, int64_t sld, int rows, int cols16,
                                          int ct, int* err) {
  if (!bounds_ok(((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u) == 0 &&
                     cols16 <= dld && cols16 <= sld && cols16 <= 32,
                 err))
    return;
  const int w = ct >> 5, lane = ct & 31;
  if (lane >= cols16) return;
  for (int r0 = w; r0 < rows; r0 += kCopyWarps * kCopyUnroll) {
    uint4 v[kCopyUnroll];
    #pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int r = r0 + u * kCopyWarps;
      if (r < rows) v[u] = ld_cg_v4(src + int64_t(r) * sld + lane);
    }
    #pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int r = r0 + u * kCopyWarps;
      if (r < rows) dst[int64_t(r) * dld + lane] = v[u];
    }
  }
}

// Copy warps: one own output tile (rows lrow0.. of this rank's chunk, global row m0..,
// columns c0..c0 + 8 ncols16) becomes y = own partial (already in y, bf16) + the peers'
// bf16 partials in ascending rank order, summed in fp32. One warp per row, one 16-byte
// vector per lane; 16 / tp rows (all their sources) loaded before the first sum, so the
// receive-buffer reads overlap. AR: each reduced row is also stored into every peer's
// output landing zone.
template <int MODE, int TP>
__device__ __forceinline__ void reduce_rows(const FusedArgs& g, const FusedPeers& p, const __nv_bfloat16* recv_tile,
                                            int64_t src_stride, int tile_ld, int lrow0, int m0, int c0, int w, int lane,
                                            int rbeg, int rend, __nv_bfloat16* ar_stage) {
  // TP: the group size, or 0 for any size up to kFusedMaxTp (one row at a time)
  constexpr int kSrc = TP > 0 ? TP : kFusedMaxTp;
  constexpr int kTpDiv = TP > 0 ? TP : 8;
  constexpr int kRows = 8 / kTpDiv > 0 ? 8 / kTpDiv : 1;  // rows whose sources load at once
  __nv_bfloat16* y = static_cast<__nv_bfloat16*>(g.c);
  for (int r0 = rbeg + w * kRows; r0 < rend; r0 += kCopyWarps * kRows) {
    uint4 v[kRows][kSrc];
    #pragma unroll
    for (int rr = 0; rr < kRows; ++rr) {
      if (r0 + rr >= rend) continue;
      const int lrow = lrow0 + r0 + rr;
      const int64_t yrow = MODE == kModeRS ? lrow : int64_t(m0 + r0 + rr);
      #pragma unroll
      for (int src = 0; src < kSrc; ++src) {
        if (TP == 0 && src >= p.tp) continue;
        const uint4* a = src == p.rank
                             ? reinterpret_cast<const uint4*>(y + yrow * g.ldc + c0) + lane
                             : reinterpret_cast<const uint4*>(recv_tile + src * src_stride +
                                                              int64_t(r0 + rr) * tile_ld) +
                                   lane;
        v[rr][src] = ld_cg_v4(a);
      }
    }
    #pragma unroll
    for (int rr = 0; rr < kRows; ++rr) {
      if (r0 + rr >= rend) continue;
      // the own partial first, then the peers' in ascending rank order
      uint4 own = v[rr][0];
      #pragma unroll
      for (int q = 1; q < kSrc; ++q)
        if (q == p.rank) own = v[rr][q];
      float tot[8];
      bf16x8_to_f32(own, tot);
      #pragma unroll
      for (int src = 0; src < kSrc; ++src) {
        if (src == p.rank || (TP == 0 && src >= p.tp)) continue;
        float x[8];
        bf16x8_to_f32(v[rr][src], x);
        #pragma unroll
        for (int e = 0; e < 8; ++e) tot[e] += x[e];
      }
      uint4 o;
      o.x = pack_bf16(tot[0], tot[1]);
      o.y = pack_bf16(tot[2], tot[3]);
      o.z = pack_bf16(tot[4], tot[5]);
      o.w = pack_bf16(tot[6], tot[7]);
      const int lrow = lrow0 + r0 + rr;
      const int64_t yrow = MODE == kModeRS ? lrow : int64_t(m0 + r0 + rr);
      reinterpret_cast<uint4*>(y + yrow * g.ldc + c0)[lane] = o;
      // AR: also into the own tile's (otherwise unused) slot of the send buffer, tile-
      // contiguous, from where the slice is bulk-pushed to every peer
      if (MODE == kModeAR) reinterpret_cast<uint4*>(ar_stage + int64_t(r0 + rr) * tile_ld)[lane] = o;
    }
  }
}

template <int MODE>
// The receive buffer is tile-contiguous: source src's partial of own tile lt starts at
// recv + (src * per_chunk + lt) * tile_elems, rows tile_ld apart.
__device__ __forceinline__ void reduce_own_tile(const FusedArgs& g, const FusedPeers& p, int lt, int per_chunk,
                                                int tile_elems, int tile_ld, int lrow0, int m0, int c0, int ncols16,
                                                int ct, int rbeg, int rend, __nv_bfloat16* ar_stage) {
  const int w = ct >> 5, lane = ct & 31;
  if (lane >= ncols16) return;
  const __nv_bfloat16* recv_tile = pick(p.recv, p.rank) + int64_t(lt) * tile_elems;
  const int64_t stride = int64_t(per_chunk) * tile_elems;
  if (p.tp == 2) reduce_rows<MODE, 2>(g, p, recv_tile, stride, tile_ld, lrow0, m0, c0, w, lane, rbeg, rend, ar_stage);
  else if (p.tp == 4) reduce_rows<MODE, 4>(g, p, recv_tile, stride, tile_ld, lrow0, m0, c0, w, lane, rbeg, rend, ar_stage);
  else reduce_rows<MODE, 0>(g, p, recv_tile, stride, tile_ld, lrow0, m0, c0, w, lane, rbeg, rend, ar_stage);
}

// One thread: ``bytes`` (a multiple of 16) from this GPU's memory at ``src`` to ``dst`` (a
// peer's memory) through the TMA engine, staged in two kChunk shared-memory buffers: the
// load of chunk c+1 overlaps the store of chunk c, and no register holds a byte in
// flight. On return every store is complete and ordered before the caller's next
// generic-proxy operations (a release on a peer's counter follows). ``phase`` carries
// the buffers' barrier phases from call to call. False if a wait ran out its budget.
__device__ __forceinline__ bool bulk_push(uint8_t* stage, uint64_t* bar, uint32_t& phase, uint8_t* dst,
                                          const uint8_t* src, int64_t bytes, int* err) {
  if (!bounds_ok(((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | uintptr_t(bytes)) & 15u) == 0,
                 err))
    return false;
  const int nch = int((bytes + kChunk - 1) / kChunk);
  bulk_wait_read_all();  // an earlier push may still be reading the buffers
  #pragma unroll 1
  for (int c = 0; c < 2 && c < nch; ++c) {
    const uint32_t len = uint32_t(min(int64_t(kChunk), bytes - int64_t(c) * kChunk));
    mbar_expect_tx(&bar[c], len);
    bulk_load(stage + c * kChunk, src + int64_t(c) * kChunk, len, &bar[c]);
  }
  bool ok = true;
  #pragma unroll 1
  for (int c = 0; c < nch; ++c) {
    const int b = c & 1;
    if (!mbar_wait(&bar[b], (phase >> b) & 1u, err, kErrEpiWait)) {
      ok = false;
      break;
    }
    phase ^= 1u << b;
    const uint32_t len = uint32_t(min(int64_t(kChunk), bytes - int64_t(c) * kChunk));
    bulk_store(dst + int64_t(c) * kChunk, stage + b * kChunk, len);
    bulk_commit();
    if (c + 2 < nch) {
      bulk_wait_read_all();  // this store has read buffer b: refill it
      const uint32_t len2 = uint32_t(min(int64_t(kChunk), bytes - int64_t(c + 2) * kChunk));
      mbar_expect_tx(&bar[b], len2);
      bulk_load(stage + b * kChunk, src + int64_t(c + 2) * kChunk, len2, &bar[b]);
    }
  }
  bulk_wait_all();
  fence_proxy_async_global();  // the async-proxy writes before the generic release that follows
  __threadfence_system();
  return ok;
}

// bulk_push without its completion wait: every chunk's store is committed as its own
// bulk group and the staging buffers are free again for the next push (the reads of all
// but the last chunk are complete; the next push waits for that one), while the writes
// may still be on their way to the peer. Used where a copy thread keeps a second push in
// flight and counts the first one only once it is complete (wait_group_keep_tile).
__device__ __forceinline__ bool bulk_push_issue(uint8_t* stage, uint64_t* bar, uint32_t& phase, uint8_t* dst,
                                                const uint8_t* src, int64_t bytes, int* err) {
  if (!bounds_ok(((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | uintptr_t(bytes)) & 15u) == 0,
                 err))
    return false;
  const int nch = int((bytes + kChunk - 1) / kChunk);
  bulk_wait_read_all();  // an earlier push may still be reading the buffers
  #pragma unroll 1
  for (int c = 0; c < 2 && c < nch; ++c) {
    const uint32_t len = uint32_t(min(int64_t(kChunk), bytes - int64_t(c) * kChunk));
    mbar_expect_tx(&bar[c], len);
    bulk_load(stage + c * kChunk, src + int64_t(c) * kChunk, len, &bar[c]);
  }
  #pragma unroll 1
  for (int c = 0; c < nch; ++c) {
    const int b = c & 1;
    if (!mbar_wait(&bar[b], (phase >> b) & 1u, err, kErrEpiWait)) return false;
    phase ^= 1u << b;
    const uint32_t len = uint32_t(min(int64_t(kChunk), bytes - int64_t(c) * kChunk));
    bulk_store(dst + int64_t(c) * kChunk, stage + b * kChunk, len);
    bulk_commit();
    if (c + 2 < nch) {
      bulk_wait_read_all();  // this store has read buffer b: refill it
      const uint32_t len2 = uint32_t(min(int64_t(kChunk), bytes - int64_t(c + 2) * kChunk));
      mbar_expect_tx(&bar[b], len2);
      bulk_load(stage + b * kChunk, src + int64_t(c + 2) * kChunk, len2, &bar[b]);
    }
  }
  return true;
}

// A whole 128 x 256 bf16 tile is four bulk groups (kChunk bytes each).
constexpr int kTileGroups = 4;
static_assert(kFBM * 256 * 2 == kTileGroups * kChunk, "an RS tile push must be kTileGroups chunks");

// Every bulk group of this thread except the kTileGroups most recent (one tile push) is
// complete: the tile pushed before the latest one has landed.
__device__ __forceinline__ void bulk_wait_keep_tile() { asm volatile("cp.async.bulk.wait_group 4;" ::: "memory"); }

// Tile t -> (chunk, m0, tn). Chunks are visited starting at (rank + first) % tp; inside a
// chunk, tiles are grouped along M (eight row blocks at a time) for L2 reuse of B.
__device__ __forceinline__ void fused_tile(int t, int tiles_m_chunk, int tiles_n, const FusedPeers& p, int first,
                                           int& chunk, int& m0, int& tn_out) {
  const int per_chunk = tiles_m_chunk * tiles_n;
  const int pos = t / per_chunk;
  const int local = t % per_chunk;
  chunk = (p.rank + first + pos) % p.tp;
  constexpr int kGroup = 8;
  const int per_group = kGroup * tiles_n;
  const int group = local / per_group;
  const int g0 = group * kGroup;
  const int size = min(tiles_m_chunk - g0, kGroup);
  const int in_group = local % per_group;
  m0 = chunk * p.rows_per_rank + (g0 + in_group % size) * kFBM;
  tn_out = in_group / size;
}

template <int BN, bool B_MN, int MODE>
__global__ void __launch_bounds__(kFusedThreads, 1)
    fused_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_land,
                      const __grid_constant__ CUtensorMap tma_b, const __grid_constant__ FusedArgs g) {
  using S = FusedShape<BN>;
  constexpr int kStages = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
  uint8_t* bstage = smem + kStages * S::kStageBytes;  // bulk-push buffers [2][kChunk]
  uint64_t* full = reinterpret_cast<uint64_t*>(bstage + 2 * kChunk);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* ring_full = acc_empty + 2;
  uint64_t* ring_empty = ring_full + kTileRing;
  int* ring = reinterpret_cast<int*>(ring_empty + kTileRing);
  int* claim = ring + kTileRing;  // copy warps: claimed item, wait outcome
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(claim + 4);
  uint64_t* bbar = reinterpret_cast<uint64_t*>(tmem_slot + 2);  // [2] bulk-push loads landed

  const FusedPeers& p = g.p;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rpr = p.rows_per_rank;
  const int tiles_m_chunk = rpr / kFBM;
  const int tiles_n = (g.n + BN - 1) / BN;
  const int per_chunk = tiles_m_chunk * tiles_n;
  const int tiles = per_chunk * p.tp;
  const int kblocks = (g.k + kFBK - 1) / kFBK;
  const int first = MODE == kModeAG ? 0 : 1;  // AG: own chunk first; RS, AR: own chunk last
  // RS counters come in two banks by call parity: contributions to one tile come from
  // tp-1 sources, and a source can be one call ahead (never two), so counting a call's
  // parity only is what keeps a fast source's next-call contributions out of this count.
  const unsigned rs_target = unsigned(p.tp - 1) * ((p.epoch + 1u) / 2u);
  unsigned* const rs_bank_local = pick(p.rs_cnt, p.rank) + (p.epoch & 1u) * kFusedMaxTiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    for (int r = 0; r < kTileRing; ++r) {
      mbar_init(&ring_full[r], 1);
      mbar_init(&ring_empty[r], 5);  // the MMA thread and the four epilogue warps
    }
    mbar_init(&bbar[0], 1);
    mbar_init(&bbar[1], 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) FUSED_STAMP(0, globaltimer());

  if (warp == 0) {
    // ---------------- tile claims + TMA producer ----------------
    if (lane == 0) {
      tma_prefetch(&tma_a);
      tma_prefetch(&tma_b);
      if (MODE == kModeAG) tma_prefetch(&tma_land);
      int s = 0;
      uint32_t ph = 0;
      int ready_key = -1;
      for (int i = 0;; ++i) {
        const int slot = i % kTileRing;
        if (!mbar_wait(&ring_empty[slot], ((i / kTileRing) & 1) ^ 1, g.err, kErrTmaWait)) break;
        int t = int(atomicAdd(p.tile_ctr, 1u) - p.tile_base);
        if (t >= tiles || t < 0) t = -1;
        ring[slot] = t;
        mbar_arrive(&ring_full[slot]);
        if (t < 0) break;
        int chunk, m0, tn;
        fused_tile(t, tiles_m_chunk, tiles_n, p, first, chunk, m0, tn);
        const int n0 = tn * BN;
        const bool own = chunk == p.rank;
        bool ok = true;
        if (MODE == kModeAG && !own) {
          const int key = chunk * kFusedMaxRb + (m0 - chunk * rpr) / kFBM;
          if (key != ready_key) {
            if (!wait_geq(p.ag_cnt[p.rank] + key, unsigned(p.slices) * p.epoch, g.err, kErrPeerWait, g.wait_ns))
              ok = false;
            fence_proxy_async_global();  // landed by peers' generic stores, read by TMA
            ready_key = key;
          }
        }
        for (int kb = 0; kb < kblocks && ok; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, g.err, kErrTmaWait)) { ok = false; break; }
          uint8_t* sa = smem + s * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_expect_tx(&full[s], S::kStageBytes);
          const int k0 = kb * kFBK;
          if (MODE == kModeAG && own) tma_load_2d(sa, &tma_a, &full[s], k0, m0 - p.rank * rpr, g.err);
          else if (MODE == kModeAG) tma_load_2d(sa, &tma_land, &full[s], k0, m0, g.err);
          else tma_load_2d(sa, &tma_a, &full[s], k0, m0, g.err);
          if (B_MN) {
            #pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_2d(sb + c * 8192, &tma_b, &full[s], n0 + 64 * c, k0, g.err);
          } else {
            tma_load_2d(sb, &tma_b, &full[s], k0, n0, g.err);
          }
          if (++s == kStages) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
      }
      FUSED_STAMP(1, globaltimer());
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kFBM, BN, 0, B_MN ? 1 : 0);
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0;; ++i) {
        const int slot = i % kTileRing;
        if (!mbar_wait(&ring_full[slot], (i / kTileRing) & 1, g.err, kErrMmaWait)) break;
        const int t = ring[slot];
        mbar_arrive(&ring_empty[slot]);
        if (t < 0) break;
        const int a = i & 1;
        const uint32_t accph = (i >> 1) & 1;
        if (!mbar_wait(&acc_empty[a], accph ^ 1, g.err, kErrMmaWait)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + a * BN;
        if (!tmem_span_ok(d, tmem_base, 2 * BN, BN, g.err)) break;
        bool ok = true;
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
        if (!ok) break;
        umma_commit(&acc_full[a]);
      }
    }
  } else if (warp < 6) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;  // this warp's TMEM lanes 32q..32q+31 = tile rows
    for (int i = 0;; ++i) {
      const int slot = i % kTileRing;
      if (!mbar_wait(&ring_full[slot], (i / kTileRing) & 1, g.err, kErrEpiWait)) break;
      const int t = ring[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&ring_empty[slot]);
      if (t < 0) break;
      int chunk, m0, tn;
      fused_tile(t, tiles_m_chunk, tiles_n, p, first, chunk, m0, tn);
      const int a = i & 1;
      const uint32_t accph = (i >> 1) & 1;
      if (!mbar_wait(&acc_full[a], accph, g.err, kErrEpiWait)) break;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const int lrow = row - chunk * rpr;
      const bool own = chunk == p.rank;
      const int local_tile = ((m0 - chunk * rpr) / kFBM) * tiles_n + tn;  // tile index inside its chunk
      bool ok = true;
      __nv_bfloat16* dst;
      if (MODE == kModeAG) dst = static_cast<__nv_bfloat16*>(g.c) + int64_t(row) * g.ldc;
      else if (!own) dst = p.send + int64_t((m0 / kFBM) * tiles_n + tn) * S::kTileElems + (row - m0) * BN - tn * BN;
      // (a peer tile's partial: local, tile-contiguous, so the copy warps push it whole)
      else if (MODE == kModeRS) dst = static_cast<__nv_bfloat16*>(g.c) + int64_t(lrow) * g.ldc;
      else dst = static_cast<__nv_bfloat16*>(g.c) + int64_t(row) * g.ldc;
      // own tiles: this rank's partial goes to y as is; the copy warps add the peers'
      // partials once they have arrived (off the MMA / epilogue critical path)
      #pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t v[32];
        const uint32_t ta = tmem_base + a * BN + cc * 32 + (uint32_t(q * 32) << 16);
        if (!tmem_span_ok(ta, tmem_base, 2 * BN, 32, g.err)) continue;
        tmem_ld32(ta, v);
        tmem_wait_ld();
        const int col0 = tn * BN + cc * 32;
        if (col0 >= g.n) continue;
        float f[32];
        #pragma unroll
        for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(v[e]);
        uint4 o[4];
        #pragma unroll
        for (int u = 0; u < 4; ++u) {
          o[u].x = pack_bf16(f[8 * u + 0], f[8 * u + 1]);
          o[u].y = pack_bf16(f[8 * u + 2], f[8 * u + 3]);
          o[u].z = pack_bf16(f[8 * u + 4], f[8 * u + 5]);
          o[u].w = pack_bf16(f[8 * u + 6], f[8 * u + 7]);
          *reinterpret_cast<uint4*>(dst + col0 + 8 * u) = o[u];
        }
      }
      if (MODE != kModeAG && !own) {
        // this warp's 32 rows of the partial tile are in the local send buffer
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(p.send_cnt + (m0 / kFBM) * tiles_n + tn, 1u);
      }
      if (MODE != kModeAG && own && ok) {
        // this warp's 32 rows of the own partial are in y: the copy warps reduce them
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(p.own_cnt + local_tile, 1u);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
      if (warp == 2 && lane == 0 && i < 8) FUSED_STAMP(2 + i, globaltimer());
    }
  } else {
    // ---------------- copy warps ----------------
    // AG items are claimed ag_copy_batch at a time; consecutive push units of one destination
    // (and consecutive gathered-copy units of one chunk) are contiguous rows, so each
    // run of a batch is one span copy, and a batch's pushes share one system fence.
    const int ct = threadIdx.x - 192;  // 0 .. kCopyThreads-1
    uint32_t bphase = 0;               // ct 0: phase bits of the two bulk-push buffers
    const int k16 = g.k / 8;           // 16-byte vectors per row of the AG input
    const int srows = kFBM / max(p.slices, 1);
    const int units = tiles_m_chunk * p.slices;  // push units of this rank's chunk (unit u = rows u*srows..)
    const int n_push = MODE == kModeAG ? (p.tp - 1) * units : 0;
    // gathered copy: every chunk into xg, or (xg is this rank's landing zone, which the
    // peers already fill) only the own chunk
    const int n_xg = MODE != kModeAG || g.xg == nullptr ? 0 : (g.xg == p.land[p.rank] ? units : p.tp * units);
    // RS / AR: push each peer-chunk partial tile to its owner (in the order the tiles are
    // claimed); AR also: push each own reduced tile to every peer, then copy the other
    // owners' reduced tiles from the output landing zone into y
    const int n_rsp = MODE != kModeAG ? (p.tp - 1) * per_chunk : 0;
    // reduce (and, AR, push) row slices of the own tiles, so the reduction spreads
    // over every CTA's copy warps
    const int red = red_slices(per_chunk, int(gridDim.x));
    const int n_own = MODE != kModeAG ? per_chunk * red : 0;
    const int n_ar = MODE == kModeAR ? (p.tp - 1) * per_chunk : 0;
    const int items = MODE == kModeAG ? n_push + n_xg : n_rsp + n_own + n_ar;
    // an RS / AR item is a whole 128 x 256 tile (or a slice of one)
    const int batch = MODE == kModeAG ? ag_copy_batch(items, int(gridDim.x)) : 1;
    // ct 0, push_depth 2: the tile counter of the last RS / AR partial push, counted
    // once the push after it is issued, or before this thread waits on a peer (a count
    // carried into such a wait can deadlock two ranks), or when the copy warps finish
    unsigned* owed = nullptr;
    auto pay_owed = [&]() {
      if (owed == nullptr) return;
      bulk_wait_all();
      fence_proxy_async_global();
      __threadfence_system();
      red_release_add(owed, 1u);
      owed = nullptr;
    };
    for (int nclaim = 0; items > 0; ++nclaim) {
      if (ct == 0) claim[0] = int(atomicAdd(p.copy_ctr, unsigned(batch)) - p.copy_base);
      copy_bar();
      const int first_item = claim[0];
      copy_bar();
      if (first_item < 0 || first_item >= items) break;
      if (ct == 0 && nclaim < 8) {
        FUSED_STAMP(10 + 2 * nclaim, globaltimer());
        FUSED_STAMP(26 + nclaim, uint64_t(first_item));
      }
      const int last_item = min(first_item + batch, items);
      bool ok = true;
      // pushes: runs of one destination, then one fence, then one count per unit
      const int pe = min(last_item, n_push);
      if (first_item < pe) {
        // one thread drives the TMA engine: each run is one contiguous span of rows
        if (ct == 0) {
          bool pushed = true;
          for (int i = first_item; i < pe && pushed;) {
            const int j = i / units;
            const int run_end = min(pe, (j + 1) * units);
            const int dest = (p.rank - j - 1 + p.tp) % p.tp;
            const int r0 = (i % units) * srows;
            pushed = bulk_push(bstage, bbar, bphase,
                               reinterpret_cast<uint8_t*>(pick(p.land, dest) + (int64_t(p.rank) * rpr + r0) * g.k),
                               reinterpret_cast<const uint8_t*>(g.x_local + int64_t(r0) * g.k),
                               int64_t(run_end - i) * srows * g.k * 2, g.err);
            i = run_end;
          }
          if (pushed)
            for (int i = first_item; i < pe; ++i) {
              const int dest = (p.rank - i / units - 1 + p.tp) % p.tp;
              red_release_add(pick(p.ag_cnt, dest) + p.rank * kFusedMaxRb + (i % units) / p.slices, 1u);
            }
          claim[1] = pushed;
        }
        copy_bar();
        ok = claim[1] != 0;
        copy_bar();
      }
      // gathered copy: runs of one chunk (own chunk first, then in arrival order)
      const int xb = max(first_item, n_push), xe = min(last_item, n_push + n_xg);
      for (int i = xb; i < xe && ok;) {
        const int i2 = i - n_push;
        const int c = (p.rank + i2 / units) % p.tp;
        const int run_end = min(xe, n_push + (i2 / units + 1) * units);
        const int u0 = i2 % units, u1 = u0 + (run_end - i);
        const __nv_bfloat16* src;
        if (c == p.rank) {
          src = g.x_local;
        } else {
          if (ct == 0) {
            int arrived = 1;
            for (int rb = u0 / p.slices; rb <= (u1 - 1) / p.slices && arrived; ++rb)
              arrived = wait_geq(p.ag_cnt[p.rank] + c * kFusedMaxRb + rb, unsigned(p.slices) * p.epoch, g.err,
                                 kErrPeerWait, g.wait_ns);
            claim[1] = arrived;
          }
          copy_bar();
          ok = claim[1] != 0;
          copy_bar();
          src = p.land[p.rank] + int64_t(c) * rpr * g.k;
        }
        if (ok)
          copy_span(reinterpret_cast<uint4*>(g.xg + (int64_t(c) * rpr + int64_t(u0) * srows) * g.k),
                    reinterpret_cast<const uint4*>(src + int64_t(u0) * srows * g.k), int64_t(u1 - u0) * srows * k16,
                    ct, g.err);
        i = run_end;
      }
      // RS / AR items (a tile, or a 16-row slice of an own tile)
      for (int it = first_item; MODE != kModeAG && it < last_item && ok; ++it) {
        int chunk, m0, tn, slice = 0;
        if (it < n_rsp) {
          fused_tile(it, tiles_m_chunk, tiles_n, p, 1, chunk, m0, tn);  // push items follow the claim order
        } else if (it < n_rsp + n_own) {
          // own tiles in their claim order (they follow the peers' tiles: t >= n_rsp)
          fused_tile(n_rsp + (it - n_rsp) / red, tiles_m_chunk, tiles_n, p, 1, chunk, m0, tn);
          slice = (it - n_rsp) % red;
        } else {
          const int i3 = it - n_rsp - n_own;  // gather: another owner's reduced tile
          chunk = (p.rank + 1 + i3 / per_chunk) % p.tp;
          const int lt = i3 % per_chunk;
          m0 = chunk * rpr + (lt / tiles_n) * kFBM;
          tn = lt % tiles_n;
        }
        const int gtile = (m0 / kFBM) * tiles_n + tn;
        const int local_tile = ((m0 - chunk * rpr) / kFBM) * tiles_n + tn;
        const int ncols16 = min(BN, g.n - tn * BN) / 8;
        if (ct == 0) {
          if (it >= n_rsp) pay_owed();  // the waits below are on peers
          if (it < n_rsp)
            claim[1] = wait_geq(p.send_cnt + gtile, 4u * p.epoch, g.err, kErrEpiWait, kWaitBudgetNs);
          else if (it < n_rsp + n_own)
            claim[1] = wait_geq(p.own_cnt + local_tile, 4u * p.epoch, g.err, kErrEpiWait, kWaitBudgetNs) &&
                       wait_geq(rs_bank_local + local_tile, rs_target, g.err, kErrPeerWait, g.wait_ns);
          else
            claim[1] = wait_geq(pick(p.ar_cnt, p.rank) + gtile, unsigned(red) * p.ar_epoch, g.err, kErrPeerWait,
                                g.wait_ns);
        }
        copy_bar();
        ok = claim[1] != 0;
        copy_bar();
        if (!ok) break;
        if (it < n_rsp) {
          // the partial tile -> the owner's receive buffer (slot of this rank): the whole
          // tile, contiguous in both buffers, through the TMA engine, then counted there
          if (ct == 0) {
            uint8_t* dst =
                reinterpret_cast<uint8_t*>(pick(p.recv, chunk) + (int64_t(p.rank) * per_chunk + local_tile) * S::kTileElems);
            const uint8_t* src = reinterpret_cast<const uint8_t*>(p.send + int64_t(gtile) * S::kTileElems);
            unsigned* cnt = pick(p.rs_cnt, chunk) + (p.epoch & 1u) * kFusedMaxTiles + local_tile;
            bool pushed;
            if (g.push_depth >= 2) {
              // issue this tile, then count the previous one once it has landed
              pushed = bulk_push_issue(bstage, bbar, bphase, dst, src, int64_t(S::kTileElems) * 2, g.err);
              if (owed != nullptr) {
                if (pushed) bulk_wait_keep_tile();
                else bulk_wait_all();
                fence_proxy_async_global();
                __threadfence_system();
                red_release_add(owed, 1u);
                owed = nullptr;
              }
              if (pushed) owed = cnt;
            } else {
              pushed = bulk_push(bstage, bbar, bphase, dst, src, int64_t(S::kTileElems) * 2, g.err);
              if (pushed) red_release_add(cnt, 1u);
            }
            claim[1] = pushed;
          }
          copy_bar();
          ok = claim[1] != 0;
          copy_bar();
        } else if (it < n_rsp + n_own) {
          // y (own partial) + every peer's partial, in rank order after the own one; AR:
          // the sum also goes to every peer's output landing zone
          const int slice_rows = kFBM / red;
          __nv_bfloat16* ar_stage = p.send + int64_t(gtile) * S::kTileElems;  // the own tile's send slot
          reduce_own_tile<MODE>(g, p, local_tile, per_chunk, S::kTileElems, BN, m0 - chunk * rpr, m0, tn * BN, ncols16,
                                ct, slice * slice_rows, (slice + 1) * slice_rows, ar_stage);
          if (MODE == kModeAR) {
            // the reduced slice (contiguous rows of the tile-contiguous stage) to every
            // peer's output landing zone (same layout) by bulk copies, then counted there
            fence_proxy_async_global();  // this thread's stage writes, before the TMA reads them
            copy_bar();
            if (ct == 0) {
              bool pushed = true;
              const int64_t off = int64_t(gtile) * S::kTileElems + int64_t(slice) * slice_rows * BN;
              #pragma unroll 1
              for (int r = 0; r < p.tp && pushed; ++r)
                if (r != p.rank)
                  pushed = bulk_push(bstage, bbar, bphase, reinterpret_cast<uint8_t*>(pick(p.out_land, r) + off),
                                     reinterpret_cast<const uint8_t*>(p.send + off), int64_t(slice_rows) * BN * 2,
                                     g.err);
              if (pushed) {
                #pragma unroll
                for (int r = 0; r < kFusedMaxTp; ++r)
                  if (r < p.tp && r != p.rank) red_release_add(p.ar_cnt[r] + gtile, 1u);
              }
              claim[1] = pushed;
            }
            copy_bar();
            ok = claim[1] != 0;
            copy_bar();
          }
        } else {
          // another owner's reduced tile: tile-contiguous landing zone -> rows of y
          copy_rows(reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(g.c) + int64_t(m0) * g.ldc + tn * BN),
                    g.ldc / 8, reinterpret_cast<const uint4*>(pick(p.out_land, p.rank) + int64_t(gtile) * S::kTileElems),
                    BN / 8, kFBM, ncols16, ct, g.err);
        }
      }
      if (ct == 0 && nclaim < 8) FUSED_STAMP(11 + 2 * nclaim, globaltimer());
      if (!ok) break;
    }
    if (ct == 0) pay_owed();
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) FUSED_STAMP(34, globaltimer());
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

uint64_t* g_fused_trace = nullptr;

int sm_count() {
  int dev = 0, n = 0;
  RESIHP_CUDA_CHECK(cudaGetDevice(&dev));
  RESIHP_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  return n;
}

template <int BN, bool B_MN, int MODE>
void launch_fused(const CUtensorMap& ta, const CUtensorMap& tl, const CUtensorMap& tb, const FusedArgs& g, int grid,
                  cudaStream_t st) {
  using S = FusedShape<BN>;
  auto kernel = fused_gemm_kernel<BN, B_MN, MODE>;
  RESIHP_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem));
  kernel<<<grid, kFusedThreads, S::kSmem, st>>>(ta, tl, tb, g);
  RESIHP_CUDA_CHECK(cudaGetLastError());
}

void check_peers(const FusedPeers& p, int t_rows, int n, int k, const char* what) {
  RESIHP_CHECK(p.tp >= 2 && p.tp <= kFusedMaxTp && p.rank >= 0 && p.rank < p.tp, what, ": bad group size / rank");
  RESIHP_CHECK(t_rows % p.tp == 0 && t_rows / p.tp == p.rows_per_rank && p.rows_per_rank % kFBM == 0, what,
               ": rows per rank must be a multiple of 128");
  RESIHP_CHECK(p.rows_per_rank / kFBM <= kFusedMaxRb, what, ": too many row blocks per rank");
  RESIHP_CHECK(n % 32 == 0 && k % 8 == 0, what, ": N must be a multiple of 32 and K of 8");
  RESIHP_CHECK((t_rows / kFBM) * ((n + 255) / 256) <= kFusedMaxTiles, what, ": too many output tiles");
  RESIHP_CHECK(p.tile_ctr != nullptr && p.copy_ctr != nullptr, what, ": missing claim counters");
}

}  // namespace

// One CTA per SM whatever the tile count: CTAs without a tile still run copy warps, and
// the bytes in flight of the pushes and copies scale with the CTAs that issue them.
int fused_grid(int m, int n, int tp) {
  (void)m;
  (void)n;
  (void)tp;
  return sm_count();
}

int fused_slices(int rows_per_rank) {
  const int blocks = std::max(1, rows_per_rank / kFBM);
  int s = 1;
  while (s < 32 && blocks * s < sm_count()) s *= 2;
  return s;
}

int fused_tile_claims(int t_rows, int n, int grid) { return (t_rows / kFBM) * ((n + 255) / 256) + grid; }

int fused_copy_claims(int mode, int t_rows, int n, int tp, int slices, int xg_chunks, int grid) {
  const int rpr = t_rows / tp;
  const int units = (rpr / kFBM) * slices;
  const int per_chunk = (rpr / kFBM) * ((n + 255) / 256);
  int items = 0;
  if (mode == kModeAG) items = (tp - 1) * units + xg_chunks * units;
  const int red = red_slices(per_chunk, grid);
  if (mode == kModeRS) items = (tp - 1) * per_chunk + per_chunk * red;
  if (mode == kModeAR) items = (tp - 1) * per_chunk + per_chunk * red + (tp - 1) * per_chunk;
  // every batch claimed, plus one failing claim per CTA, a batch of items each
  const int batch = mode == kModeAG ? ag_copy_batch(items, grid) : 1;
  return items > 0 ? ((items + batch - 1) / batch + grid) * batch : 0;
}

int fused_red_slices(int t_rows, int n, int tp, int grid) {
  return red_slices((t_rows / tp / kFBM) * ((n + 255) / 256), grid);
}

void set_fused_trace(uint64_t* buffer) { g_fused_trace = buffer; }

int fused_trace_slots() { return kTraceSlots; }

void fused_ag_gemm(const void* x_local, void* xg, const void* w, int64_t ldw, bool w_mn, void* y, int64_t ldy,
                   int t_rows, int n, int k, const FusedPeers& peers, int grid, int* err, cudaStream_t st) {
  check_peers(peers, t_rows, n, k, "ag_gemm");
  RESIHP_CHECK(peers.slices >= 1 && peers.slices <= 32 && (peers.slices & (peers.slices - 1)) == 0,
               "ag_gemm: push slices must be a power of two up to 32");
  for (int r = 0; r < peers.tp; ++r)
    RESIHP_CHECK(peers.land[r] != nullptr && peers.ag_cnt[r] != nullptr, "ag_gemm: missing peer buffers");
  const int tl = t_rows / peers.tp;
  CUtensorMap ta = make_tma_2d_bf16(x_local, tl, k, k, 64, kFBM);
  CUtensorMap tland = make_tma_2d_bf16(peers.land[peers.rank], t_rows, k, k, 64, kFBM);
  CUtensorMap tb = w_mn ? make_tma_2d_bf16(w, k, n, ldw, 64, 64) : make_tma_2d_bf16(w, n, k, ldw, 64, 256);
  FusedArgs g{};
  g.c = y;
  g.ldc = ldy;
  g.m = t_rows;
  g.n = n;
  g.k = k;
  g.err = err;
  g.wait_ns = peer_wait_budget_ns();
  g.trace = g_fused_trace;
  g.x_local = static_cast<const __nv_bfloat16*>(x_local);
  g.xg = static_cast<__nv_bfloat16*>(xg);
  g.p = peers;
  if (w_mn) launch_fused<256, true, kModeAG>(ta, tland, tb, g, grid, st);
  else launch_fused<256, false, kModeAG>(ta, tland, tb, g, grid, st);
}

// RESIHP_PUSH_DEPTH=2: RS / AR partial-tile pushes pipelined two deep per copy thread
// (each counted once the next is issued); default 1, one push completed at a time.
static int g_push_depth = [] {
  const char* e = std::getenv("RESIHP_PUSH_DEPTH");
  return e != nullptr && e[0] == '2' ? 2 : 1;
}();

void set_fused_push_depth(int depth) { g_push_depth = depth >= 2 ? 2 : 1; }

void fused_gemm_rs(const void* h, const void* w, int64_t ldw, bool w_mn, void* y, int64_t ldy, int t_rows, int n,
                   int k, bool all_reduce, const FusedPeers& peers, int grid, int* err, cudaStream_t st) {
  check_peers(peers, t_rows, n, k, all_reduce ? "gemm_ar" : "gemm_rs");
  for (int r = 0; r < peers.tp; ++r) {
    RESIHP_CHECK(peers.recv[r] != nullptr && peers.rs_cnt[r] != nullptr, "gemm_rs: missing peer buffers");
    RESIHP_CHECK(!all_reduce || (peers.out_land[r] != nullptr && peers.ar_cnt[r] != nullptr),
                 "gemm_ar: missing peer output buffers");
  }
  CUtensorMap ta = make_tma_2d_bf16(h, t_rows, k, k, 64, kFBM);
  CUtensorMap tb = w_mn ? make_tma_2d_bf16(w, k, n, ldw, 64, 64) : make_tma_2d_bf16(w, n, k, ldw, 64, 256);
  FusedArgs g{};
  g.c = y;
  g.ldc = ldy;
  g.m = t_rows;
  g.n = n;
  g.k = k;
  g.err = err;
  g.wait_ns = peer_wait_budget_ns();
  g.trace = g_fused_trace;
  g.push_depth = g_push_depth;
  g.p = peers;
  if (all_reduce) {
    if (w_mn) launch_fused<256, true, kModeAR>(ta, ta, tb, g, grid, st);
    else launch_fused<256, false, kModeAR>(ta, ta, tb, g, grid, st);
  } else {
    if (w_mn) launch_fused<256, true, kModeRS>(ta, ta, tb, g, grid, st);
    else launch_fused<256, false, kModeRS>(ta, ta, tb, g, grid, st);
  }
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
