// Torch-free host interface of the CUDA kernels. Each launcher validates its arguments,
// enqueues on ``stream`` and throws std::runtime_error on misuse; the torch-facing
// wrappers in torch_api.cpp translate tensors into these calls. No counterpart in the
// reference, which has no native code.
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace resihp {

// Error messages are assembled with std::string / std::to_string only (no iostreams):
// they must be safe to build on any thread, including autograd worker threads.
namespace detail {
inline void append(std::string&) {}
template <class T, class... R>
inline void append(std::string& o, const T& v, const R&... r) {
  if constexpr (std::is_arithmetic_v<T>) o += std::to_string(v);
  else o += v;
  append(o, r...);
}
}  // namespace detail

#define RESIHP_CHECK(cond, ...)                                                        \
  do {                                                                                 \
    if (!(cond)) {                                                                     \
      std::string _o;                                                                  \
      ::resihp::detail::append(_o, "resihp: ", __VA_ARGS__);                           \
      throw std::runtime_error(_o);                                                    \
    }                                                                                  \
  } while (0)

#define RESIHP_CUDA_CHECK(expr)                                                        \
  do {                                                                                 \
    cudaError_t _e = (expr);                                                           \
    RESIHP_CHECK(_e == cudaSuccess, #expr, " failed: ", cudaGetErrorString(_e));        \
  } while (0)

// Budget of every wait on another GPU's flag inside a kernel, in nanoseconds (default
// 4 s). The host reads it at each launch of a kernel that waits on peers and passes it
// as a launch argument; a wait that runs out records kErrPeerWait in the device's error
// word and the kernel returns. Tests shorten it to make a wait that nothing completes
// end quickly.
uint64_t peer_wait_budget_ns();
void set_peer_wait_budget_ns(uint64_t ns);

// AdamW coefficients of one step (bias corrections folded in on the host, in double).
struct AdamWCoef {
  float lr, b1, b2, eps, wd, step_size, bc2_sqrt, grad_scale;
};
AdamWCoef adamw_coef(float lr, float b1, float b2, float eps, float wd, int64_t step, float grad_scale);

CUtensorMap make_tma_2d_bf16(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_cols, int box_rows);

// C[m,n] (=, +=) alpha * A * B^T; see gemm.cu for operand conventions and epilogues.
void gemm_raw(const void* a, int64_t lda, bool a_mn, const void* b, int64_t ldb, bool b_mn, void* c, int64_t ldc,
              const void* r, int64_t ldr, int m, int n, int k, int epi, float alpha, int* err, cudaStream_t stream,
              int max_ctas, int force_bn);

}  // namespace resihp

namespace resihp {

int rmsnorm_partial_rows(int rows, int d, int num_sms);
void rmsnorm_fwd(const void* x, const void* r, const void* w, void* y, void* s_out, float* rstd, int rows, int d,
                 float eps, int num_sms, cudaStream_t st);
void rmsnorm_bwd(const void* dy, const void* s, const void* w, const float* rstd, const void* dres, void* ds,
                 float* partial, float* dw, int accumulate, int rows, int d, int num_sms, cudaStream_t st);

void rope(void* qkv, const float* cs, int rows, int seq, int heads_qk, int hd, int64_t row_stride, int pos_offset,
          bool inverse, int num_sms, cudaStream_t st);
void swiglu_fwd(const void* gu, void* h, int rows, int f, int num_sms, cudaStream_t st);
void swiglu_bwd(const void* gu, const void* dh, void* dgu, int rows, int f, int num_sms, cudaStream_t st);
void adamw(float* p, const float* g, float* m, float* v, void* p_bf16, int64_t n, float lr, float b1, float b2,
           float eps, float wd, int64_t step, float grad_scale, int num_sms, cudaStream_t st);
void embedding_fwd(const int64_t* ids, const void* w, void* out, int rows, int d, int64_t start, int64_t count,
                   cudaStream_t st);
// keys: device scratch of min(rows, embedding_sort_segment()) uint64 values.
int embedding_sort_segment();
void embedding_bwd(const int64_t* ids, const void* dy, float* dw, uint64_t* keys, int rows, int d, int64_t start,
                   int64_t count, cudaStream_t st);

void xent_stats(const void* logits, int64_t ld, const int64_t* labels, float* stats, int rows, int v, int64_t start,
                cudaStream_t st);
void xent_grad(void* logits, int64_t ld, const int64_t* labels, const float* lse, const float* scale, int rows, int v,
               int64_t start, cudaStream_t st);

void attn_fwd(const void* qkv, int64_t qkv_ld, void* out, int64_t out_ld, float* lse, int rows, int seq, int hq,
              int hkv, int d, float scale, int* err, cudaStream_t st);
void attn_bwd(const void* qkv, int64_t qkv_ld, const void* out, int64_t out_ld, const void* dout, int64_t dout_ld,
              const float* lse, float* delta, void* dqkv, int64_t dqkv_ld, int rows, int seq, int hq, int hkv, int d,
              float scale, int* err, cudaStream_t st);

}  // namespace resihp

namespace resihp {

// Fused TP collectives (fused_gemm.cu). Every rank of a TP group maps every other
// rank's symmetric workspace; these are this call's pointers into all of them.
constexpr int kFusedMaxTp = 8;
constexpr int kFusedMaxRb = 256;      // 128-row blocks per rank's chunk
constexpr int kFusedMaxTiles = 8192;  // output tiles (128 x 256) per call
struct FusedPeers {
  int rank, tp, rows_per_rank;
  int slices;              // AG push units per 128-row block (a power of two up to 32)
  unsigned epoch;          // AG: AG calls so far (this one included); RS, AR: RS + AR calls
  unsigned ar_epoch;       // AR calls so far
  unsigned* tile_ctr;      // local work-claim counters and the values they had before this call
  unsigned tile_base;
  unsigned* copy_ctr;
  unsigned copy_base;
  __nv_bfloat16* land[kFusedMaxTp];      // AG landing zone [T, K] of each rank (this call's parity)
  unsigned* ag_cnt[kFusedMaxTp];         // AG counters [kFusedMaxTp][kFusedMaxRb] of each rank
  __nv_bfloat16* recv[kFusedMaxTp];      // RS receive buffer [tp][T/tp, N] of each rank (parity)
  unsigned* rs_cnt[kFusedMaxTp];         // RS per-own-tile counters [2 parities][kFusedMaxTiles] of each rank
  __nv_bfloat16* out_land[kFusedMaxTp];  // AR reduced-output landing zone [T, N] of each rank (parity)
  unsigned* ar_cnt[kFusedMaxTp];         // AR per-tile counters of each rank
  __nv_bfloat16* send;                   // local: RS partial tiles [T, N] before the push
  unsigned* send_cnt;                    // local: per-tile count of finished partial rows (4 warps per call)
  unsigned* own_cnt;                     // local: per-own-tile count of finished reduced rows (AR)
};
int fused_grid(int m, int n, int tp);
int fused_slices(int rows_per_rank);
// Claims a launch makes on its counters (the host adds them to its bases after the call).
int fused_tile_claims(int t_rows, int n, int grid);
// xg_chunks: chunks copied into the gathered input (0: none, 1: only the own chunk into
// this rank's landing zone, tp: every chunk into a separate buffer).
int fused_copy_claims(int mode, int t_rows, int n, int tp, int slices, int xg_chunks, int grid);
// Row slices per own tile in the RS / AR reduction (the AR counts each slice).
int fused_red_slices(int t_rows, int n, int tp, int grid);
// Profiling aid: stamp per-CTA timelines of the fused kernels into ``buffer``
// ([grid][fused_trace_slots()] uint64 device memory), or stop (nullptr).
void set_fused_trace(uint64_t* buffer);
int fused_trace_slots();
// RS / AR partial-tile pushes pipelined two deep per copy thread (2) or one at a time (1).
void set_fused_push_depth(int depth);
void fused_ag_gemm(const void* x_local, void* xg, const void* w, int64_t ldw, bool w_mn, void* y, int64_t ldy,
                   int t_rows, int n, int k, const FusedPeers& peers, int grid, int* err, cudaStream_t st);
void fused_gemm_rs(const void* h, const void* w, int64_t ldw, bool w_mn, void* y, int64_t ldy, int t_rows, int n,
                   int k, bool all_reduce, const FusedPeers& peers, int grid, int* err, cudaStream_t st);
void* symm_alloc(int64_t bytes, void* handle_out);
void* symm_open(const void* handle);
void symm_close(void* p);
void symm_free(void* p);

}  // namespace resihp

namespace resihp {

// Peer-memory kernels over a stage's flat training state (peer_state.cu).
constexpr int kMaxDp = 8;
int dp_grid(int64_t n, int num_sms);
// One-phase (sums_peer == nullptr): every rank reads every peer's whole accumulated
// gradient. Two-phase push variant (sums_peer, flags2_*): rank q reduces part q of each
// CTA slice, pushes the sum into every rank's receiving buffer, then steps locally.
void dp_allreduce_adamw(const float* const* grads, int dp, int me, float* sum_out, float* p, float* m, float* v,
                        void* p_bf16, int64_t n, const AdamWCoef& coef, unsigned* flags_local,
                        unsigned* const* flags_peer, unsigned epoch, int grid, int* err, cudaStream_t st,
                        float* const* sums_peer = nullptr, unsigned* flags2_local = nullptr,
                        unsigned* const* flags2_peer = nullptr);

// One strided block copy of the state move: rows x cols fp32 elements.
struct CopyDesc {
  const float* src;
  float* dst;
  void* dst_bf16;     // optional bf16 copy at the same element offsets (the compute weights)
  int64_t src_ld, dst_ld;
  int64_t rows, cols;
  int64_t item_base;  // first work item (one item = one row) of this descriptor
  int64_t vec4;       // 1: every address, stride and width is a multiple of 16 bytes
};
void reshard_gather(const CopyDesc* descs_device, int ndesc, int64_t items, int* err, int num_sms, cudaStream_t st);

}  // namespace resihp
