// Shared sm_100a device helpers: mbarriers with bounded waits, TMA tile loads and bulk
// copies, the tcgen05 (5th-generation tensor core + tensor memory) instructions the
// kernels use, and programmatic dependent launch (launch_pdl / pdl_enter).
//
// Every spin-wait here is bounded by the global nanosecond timer. A wait that runs out
// records a code in the kernel's error word and returns false; the caller then leaves
// its loop, so a kernel can never hang the GPU on a barrier that is never completed.
// The host reads the error word after the launch and raises. (No counterpart in the
// reference, which runs library kernels only.)
#pragma once
#include <cstdint>
#include <cstdlib>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "launch.h"

namespace resihp {

// Wait budget for one barrier phase. Generous on purpose: a healthy wait is
// microseconds; this only has to be short enough to turn a bug into an error. Waits on
// another GPU's flags take their budget from the launch instead (``peer_wait_budget_ns``
// on the host, default the same 4 s), so a test can make such a wait run out quickly.
constexpr uint64_t kWaitBudgetNs = 4000000000ull;

enum ErrorCode : int {
  kErrNone = 0,
  kErrTmaWait = 1,      // producer waited too long for a free smem stage
  kErrMmaWait = 2,      // MMA issuer waited too long for a filled stage / free accumulator
  kErrEpiWait = 3,      // epilogue waited too long for a finished accumulator
  kErrPeerWait = 4,     // a cross-GPU flag never arrived
  kErrBounds = 5,       // a bounds check in a checked build skipped an access
};

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// ---- bounds-checked build ---------------------------------------------------------------
// Compiled with -DRESIHP_BOUNDS_CHECK (the separate library ``_C_checked.so``), the
// kernels test the addresses they compute before they use them: TMA tile coordinates
// (innermost coordinate on a 16-byte boundary, no negative coordinate, shared-memory
// destination on the 1024-byte swizzle boundary), TMEM column ranges against the
// allocation, offsets into shared-memory tiles against the tile, and element offsets
// into peer buffers against the buffer. A failed test records kErrBounds in the kernel's
// error word and the access is skipped; a wait that depended on it runs out its budget
// and the kernel returns. In the default build every test is a compile-time ``true``.
#ifdef RESIHP_BOUNDS_CHECK
constexpr bool kBoundsCheck = true;
#else
constexpr bool kBoundsCheck = false;
#endif

__device__ __forceinline__ bool bounds_ok(bool ok, int* err) {
  if constexpr (kBoundsCheck) {
    if (!ok) {
      record_error(err, kErrBounds);
      return false;
    }
  }
  return true;
}

// A ``width``-column TMEM access at ``taddr`` stays inside the ``ncols`` columns
// allocated at ``base`` (and in lanes 0..127).
__device__ __forceinline__ bool tmem_span_ok(uint32_t taddr, uint32_t base, uint32_t ncols, uint32_t width,
                                             int* err) {
  const uint32_t col = (taddr & 0xFFFFu) - (base & 0xFFFFu);
  return bounds_ok((taddr >> 16) < 128u && col + width <= ncols, err);
}

// ---- programmatic dependent launch ---------------------------------------------------
// A kernel launched by launch_pdl may be scheduled while the previous kernel of its stream
// is still finishing (its launch and CTA placement overlap that kernel's tail), so every
// such kernel begins with pdl_enter(): griddepcontrol.wait blocks until the previous
// kernel has completed and its memory operations are visible (before this kernel touches
// global memory), then griddepcontrol.launch_dependents lets the next kernel of the
// stream be scheduled the same way. Launched normally, both instructions do nothing.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// RESIHP_PDL=0 launches every kernel with full stream serialisation instead.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("RESIHP_PDL");
    return e == nullptr || e[0] != '0';
  }();
  return on;
}

// <<<grid, block, smem, st>>> with programmatic stream serialisation allowed (the kernel
// must start with pdl_enter()); the launch error is returned, not raised.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---- mbarrier ------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete; false (and an error code) if
// the budget runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  const uint32_t b = smem_u32(bar);
  #pragma unroll 1
  for (int i = 0; i < 128; ++i)
    if (mbar_try_wait(b, parity)) return true;
  const uint64_t start = globaltimer();
  #pragma unroll 1
  while (true) {
    if (mbar_try_wait(b, parity)) return true;
    if (globaltimer() - start > kWaitBudgetNs) {
      record_error(err, code);
      return false;
    }
  }
}

// ---- TMA -------------------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load into this CTA's shared memory; completion is counted on ``bar``.
// ``x`` is the innermost coordinate; callers keep x * sizeof(elem) a multiple of 16.
// Every tensor map of this package holds bf16, so the checked build tests x % 8.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int* err = nullptr) {
  if (!bounds_ok((x & 7) == 0 && x >= 0 && y >= 0 && (smem_u32(dst) & 1023u) == 0, err)) return;
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int* err = nullptr) {
  if (!bounds_ok((x & 7) == 0 && x >= 0 && y >= 0 && z >= 0 && (smem_u32(dst) & 1023u) == 0, err)) return;
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ---- tcgen05 ---------------------------------------------------------------------------

// Allocate ``ncols`` TMEM columns (power of two >= 32); the base address lands in smem.
// Must be executed by one whole warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulate; one thread issues.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T (A operand read from tensor memory).
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on ``bar`` once every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
// a_mn / b_mn: operand is MN-major in shared memory (0 = K-major).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n, int a_mn, int b_mn) {
  return (1u << 4)                      // D format: f32
         | (1u << 7)                    // A format: bf16
         | (1u << 10)                   // B format: bf16
         | (uint32_t(a_mn) << 15)       // A major
         | (uint32_t(b_mn) << 16)       // B major
         | (uint32_t(n >> 3) << 17)     // N / 8
         | (uint32_t(m >> 4) << 24);    // M / 16
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm_100 version 1.
// ``lbo``/``sbo`` are byte offsets (multiples of 16).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((saddr & 0x3FFFF) >> 4);
  d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFF) << 32;
  d |= uint64_t(1) << 46;   // descriptor version for sm_100
  d |= uint64_t(2) << 61;   // SWIZZLE_128B
  return d;
}

// 32 lanes x 32 consecutive 32-bit TMEM columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---- bulk asynchronous copies (TMA engine, 1-D, no multicast) --------------------------

// ``bytes`` (a multiple of 16, both addresses 16-byte aligned) from global memory of this
// GPU into this CTA's shared memory; completion is counted on ``bar``.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// ``bytes`` from this CTA's shared memory to global memory (this GPU's or a peer's),
// added to the thread's current bulk group.
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}

// Start bringing ``bytes`` (a multiple of 16, 16-byte aligned) of this GPU's global memory
// into L2; nothing waits for it, and no shared memory or barrier is involved.
__device__ __forceinline__ void l2_prefetch_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Every committed bulk group of this thread has finished reading its shared memory.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Every committed bulk group of this thread is complete (its writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---- CTA pairs (tcgen05 cta_group::2) ----------------------------------------------
// Two CTAs of a 2-CTA cluster share one MMA: the even CTA (the leader) issues
// tcgen05.mma.cta_group::2, which reads the A and B halves from both CTAs' shared memory
// at the same offsets and writes each CTA's half of the accumulator into its own TMEM.
// All tcgen05 allocation / MMA / commit instructions of such a kernel use cta_group::2.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of both CTAs: release this CTA's prior writes, acquire the peer's.
// (Per-thread form: callable where a warp's lanes arrive at different times.)
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// shared::cluster address of this CTA's shared-memory object ``p`` as seen in CTA ``rank``.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

// Arrive on an mbarrier of another CTA of the cluster (release at cluster scope).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// mbar_wait with acquire at cluster scope, for a barrier that CTAs of the cluster arrive on.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err, int code) {
  const uint32_t b = smem_u32(bar);
  const uint64_t start = globaltimer();
  #pragma unroll 1
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(b), "r"(parity)
        : "memory");
    if (ok) return true;
    if (globaltimer() - start > kWaitBudgetNs) {
      record_error(err, code);
      return false;
    }
  }
}

// 2-D tiled load into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (``bar_cluster``: a shared::cluster address).
// No multicast: each CTA loads its own half.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y,
                                                 int* err = nullptr) {
  if (!bounds_ok((x & 7) == 0 && x >= 0 && y >= 0 && (smem_u32(dst) & 1023u) == 0, err)) return;
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

// Called by the same warp of both CTAs: ``ncols`` TMEM columns in each, at one address.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Leader only: D[tmem of both CTAs] (+)= A * B^T over the pair (M = 256 split by CTA,
// N split by CTA for the operand, whole N in each CTA's accumulator).
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Leader only: arrive once on the mbarrier at ``bar_cluster`` (either CTA) when every
// pair MMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- cross-GPU flag words (system scope) ---------------------------------------------

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

__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until *p >= target (wrap-safe); false + error code when ``budget_ns`` runs out.
// The counter is polled with relaxed loads (a short sleep between polls once the first
// few miss, so a waiting thread does not crowd the memory system its SM's other warps
// use) and the acquire is one fence after the condition holds.
__device__ __forceinline__ bool wait_geq(const unsigned* p, unsigned target, int* err, int code, uint64_t budget_ns) {
  if (static_cast<int>(ld_acquire_sys(p) - target) >= 0) return true;
  const uint64_t start = globaltimer();
  #pragma unroll 1
  for (int i = 0; static_cast<int>(ld_relaxed_sys(p) - target) < 0; ++i) {
    if (i >= 8) __nanosleep(128);
    if (globaltimer() - start > budget_ns) {
      record_error(err, code);
      return false;
    }
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  return true;
}

// ---- AdamW, one element (torch.optim.AdamW's formulation) -----------------------------
// Shared by the stand-alone optimizer kernel and the fused DP-reduce + AdamW kernel, so
// both paths round identically.
__device__ __forceinline__ void adamw_elem(float& p, float& m, float& v, float g, const AdamWCoef& c) {
  const float gi = g * c.grad_scale;
  float pi = p * (1.f - c.lr * c.wd);
  const float mi = m + (1.f - c.b1) * (gi - m);
  const float vi = c.b2 * v + (1.f - c.b2) * gi * gi;
  const float denom = sqrtf(vi) / c.bc2_sqrt + c.eps;
  pi = pi - c.step_size * (mi / denom);
  p = pi;
  m = mi;
  v = vi;
}

}  // namespace resihp
