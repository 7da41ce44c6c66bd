// Torch-facing wrappers and Python bindings of the sm_100a kernels (module resihp._C).
// Shapes, dtypes and strides are checked here; the CUDA launchers behind launch.h only
// see raw pointers, so the kernel translation units stay free of torch headers.
// (The reference is pure Python and calls torch / NCCL ops directly; this layer has no
// counterpart there.)
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>
#include <csignal>
#include <execinfo.h>
#include <unistd.h>

#include "launch.h"

namespace resihp {

// ---- error word ---------------------------------------------------------------------

static int* g_error_words[64] = {nullptr};
static std::mutex g_error_mutex;

int* error_word(const c10::Device& device) {
  const int idx = device.index() < 0 ? 0 : device.index();
  TORCH_CHECK(idx < 64, "device index out of range");
  if (g_error_words[idx] == nullptr) {
    std::lock_guard<std::mutex> lock(g_error_mutex);
    if (g_error_words[idx] == nullptr) {
      c10::cuda::CUDAGuard guard(device);
      int* p = nullptr;
      C10_CUDA_CHECK(cudaMalloc(&p, sizeof(int)));
      C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
      g_error_words[idx] = p;
    }
  }
  return g_error_words[idx];
}

// Synchronising read of the device's error word; resets it to zero.
int64_t read_and_clear_error(int64_t device_index) {
  const c10::Device dev(c10::kCUDA, device_index);
  int* p = error_word(dev);
  c10::cuda::CUDAGuard guard(dev);
  auto stream = at::cuda::getCurrentCUDAStream();
  int value = 0;
  C10_CUDA_CHECK(cudaMemcpyAsync(&value, p, sizeof(int), cudaMemcpyDeviceToHost, stream));
  C10_CUDA_CHECK(cudaStreamSynchronize(stream));
  if (value != 0) C10_CUDA_CHECK(cudaMemsetAsync(p, 0, sizeof(int), stream));
  return value;
}

static cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

static void check_cuda_bf16(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bf16");
}

// ---- GEMM ---------------------------------------------------------------------------

void gemm(torch::Tensor a, bool a_mn, torch::Tensor b, bool b_mn, torch::Tensor c, int64_t epi, double alpha,
          c10::optional<torch::Tensor> residual, int64_t max_ctas, int64_t force_bn) {
  check_cuda_bf16(a, "A");
  check_cuda_bf16(b, "B");
  TORCH_CHECK(c.is_cuda(), "C must be a CUDA tensor");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "GEMM operands must be 2-D");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && c.stride(1) == 1, "GEMM operands need unit inner stride");
  const int64_t m = a_mn ? a.size(1) : a.size(0);
  const int64_t k = a_mn ? a.size(0) : a.size(1);
  const int64_t n = b_mn ? b.size(1) : b.size(0);
  const int64_t kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(k == kb, "GEMM reduction sizes differ: ", k, " vs ", kb);
  TORCH_CHECK(c.size(0) == m && c.size(1) == n, "GEMM output shape mismatch");
  TORCH_CHECK(epi >= 0 && epi <= 4, "unknown GEMM epilogue ", epi);
  const bool want_f32 = epi == 1 || epi == 2 || epi == 4;
  TORCH_CHECK(c.scalar_type() == (want_f32 ? at::kFloat : at::kBFloat16), "GEMM output dtype does not match epilogue");
  const void* r = nullptr;
  int64_t ldr = 0;
  if (epi == 3) {
    TORCH_CHECK(residual.has_value(), "residual epilogue needs a residual tensor");
    const auto& rt = *residual;
    check_cuda_bf16(rt, "residual");
    TORCH_CHECK(rt.size(0) == m && rt.size(1) == n && rt.stride(1) == 1, "residual must be [m, n]");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(rt.data_ptr()) % 16 == 0 && rt.stride(0) % 8 == 0, "residual alignment");
    r = rt.data_ptr();
    ldr = rt.stride(0);
  }
  TORCH_CHECK(m <= INT32_MAX && n <= INT32_MAX && k <= INT32_MAX, "GEMM too large");
  c10::cuda::CUDAGuard guard(a.device());
  gemm_raw(a.data_ptr(), a.stride(0), a_mn, b.data_ptr(), b.stride(0), b_mn, c.data_ptr(), c.stride(0), r, ldr,
           int(m), int(n), int(k), int(epi), float(alpha), error_word(a.device()), cur_stream(), int(max_ctas),
           int(force_bn));
}


static int sms(const torch::Tensor& t) {
  static int counts[64] = {0};
  const int dev = t.device().index();
  if (counts[dev] == 0) C10_CUDA_CHECK(cudaDeviceGetAttribute(&counts[dev], cudaDevAttrMultiProcessorCount, dev));
  return counts[dev];
}

static void check_rows(const torch::Tensor& t, int64_t cols, const char* name) {
  check_cuda_bf16(t, name);
  TORCH_CHECK(t.dim() == 2 && t.size(1) == cols && t.is_contiguous(), name, " must be contiguous [rows, ", cols, "]");
}

// ---- RMSNorm --------------------------------------------------------------------------

std::vector<torch::Tensor> rmsnorm_fwd_t(torch::Tensor x, c10::optional<torch::Tensor> r, torch::Tensor w, double eps) {
  const int64_t d = w.numel();
  check_rows(x, d, "x");
  check_cuda_bf16(w, "w");
  c10::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({x.size(0)}, x.options().dtype(torch::kFloat));
  torch::Tensor s = x;
  const void* rp = nullptr;
  if (r.has_value()) {
    check_rows(*r, d, "residual");
    s = torch::empty_like(x);
    rp = r->data_ptr();
  }
  rmsnorm_fwd(x.data_ptr(), rp, w.data_ptr(), y.data_ptr(), rp ? s.data_ptr() : nullptr, rstd.data_ptr<float>(),
              int(x.size(0)), int(d), float(eps), sms(x), cur_stream());
  return {y, s, rstd};
}

torch::Tensor rmsnorm_bwd_t(torch::Tensor dy, torch::Tensor s, torch::Tensor w, torch::Tensor rstd,
                            c10::optional<torch::Tensor> dres, torch::Tensor dw, bool accumulate) {
  const int64_t d = w.numel();
  check_rows(dy, d, "dy");
  check_rows(s, d, "s");
  TORCH_CHECK(dw.scalar_type() == torch::kFloat && dw.numel() == d && dw.is_contiguous(), "dw must be fp32 [d]");
  c10::cuda::CUDAGuard guard(dy.device());
  const int rows = int(dy.size(0));
  auto partial = torch::empty({rmsnorm_partial_rows(rows, int(d), sms(dy)), d}, dy.options().dtype(torch::kFloat));
  auto ds = torch::empty_like(dy);
  const void* dr = nullptr;
  if (dres.has_value()) {
    check_rows(*dres, d, "dres");
    dr = dres->data_ptr();
  }
  rmsnorm_bwd(dy.data_ptr(), s.data_ptr(), w.data_ptr(), rstd.data_ptr<float>(), dr, ds.data_ptr(),
              partial.data_ptr<float>(), dw.data_ptr<float>(), accumulate ? 1 : 0, rows, int(d), sms(dy), cur_stream());
  return ds;
}

// ---- RoPE / SwiGLU --------------------------------------------------------------------

void rope_t(torch::Tensor qkv, torch::Tensor cs, int64_t seq, int64_t heads_qk, int64_t hd, int64_t pos_offset,
            bool inverse) {
  check_cuda_bf16(qkv, "qkv");
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1, "qkv must be 2-D with unit inner stride");
  TORCH_CHECK(cs.scalar_type() == torch::kFloat && cs.is_contiguous() && cs.numel() == seq * hd, "cs must be fp32 [seq, hd/2, 2]");
  c10::cuda::CUDAGuard guard(qkv.device());
  rope(qkv.data_ptr(), cs.data_ptr<float>(), int(qkv.size(0)), int(seq), int(heads_qk), int(hd), qkv.stride(0),
       int(pos_offset), inverse, sms(qkv), cur_stream());
}

torch::Tensor swiglu_fwd_t(torch::Tensor gu) {
  check_cuda_bf16(gu, "gu");
  TORCH_CHECK(gu.dim() == 2 && gu.is_contiguous(), "gu must be contiguous [rows, 2F]");
  c10::cuda::CUDAGuard guard(gu.device());
  const int64_t f = gu.size(1) / 2;
  auto h = torch::empty({gu.size(0), f}, gu.options());
  swiglu_fwd(gu.data_ptr(), h.data_ptr(), int(gu.size(0)), int(f), sms(gu), cur_stream());
  return h;
}

torch::Tensor swiglu_bwd_t(torch::Tensor gu, torch::Tensor dh) {
  check_cuda_bf16(gu, "gu");
  const int64_t f = gu.size(1) / 2;
  check_rows(dh, f, "dh");
  c10::cuda::CUDAGuard guard(gu.device());
  auto dgu = torch::empty_like(gu);
  swiglu_bwd(gu.data_ptr(), dh.data_ptr(), dgu.data_ptr(), int(gu.size(0)), int(f), sms(gu), cur_stream());
  return dgu;
}

// ---- AdamW ----------------------------------------------------------------------------

void adamw_t(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, c10::optional<torch::Tensor> p_bf16,
             double lr, double b1, double b2, double eps, double wd, int64_t step, double grad_scale) {
  for (auto* t : {&p, &g, &m, &v})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat && t->is_contiguous() && t->numel() == p.numel(),
                "AdamW buffers must be contiguous fp32 of equal size");
  void* pb = nullptr;
  if (p_bf16.has_value()) {
    TORCH_CHECK(p_bf16->scalar_type() == torch::kBFloat16 && p_bf16->numel() == p.numel() && p_bf16->is_contiguous(),
                "bf16 copy must match");
    pb = p_bf16->data_ptr();
  }
  c10::cuda::CUDAGuard guard(p.device());
  adamw(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), pb, p.numel(), float(lr),
        float(b1), float(b2), float(eps), float(wd), step, float(grad_scale), sms(p), cur_stream());
}

// ---- embedding ------------------------------------------------------------------------

torch::Tensor embedding_fwd_t(torch::Tensor ids, torch::Tensor w, int64_t start) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == torch::kLong && ids.is_contiguous(), "ids must be int64 CUDA");
  check_cuda_bf16(w, "w");
  TORCH_CHECK(w.dim() == 2 && w.is_contiguous(), "embedding table must be contiguous");
  c10::cuda::CUDAGuard guard(w.device());
  auto out = torch::empty({ids.numel(), w.size(1)}, w.options());
  embedding_fwd(ids.data_ptr<int64_t>(), w.data_ptr(), out.data_ptr(), int(ids.numel()), int(w.size(1)), start,
                w.size(0), cur_stream());
  return out;
}

void embedding_bwd_t(torch::Tensor ids, torch::Tensor dy, torch::Tensor dw, int64_t start) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == torch::kLong, "ids must be int64 CUDA");
  check_cuda_bf16(dy, "dy");
  TORCH_CHECK(dw.scalar_type() == torch::kFloat && dw.dim() == 2 && dw.is_contiguous(), "dw must be fp32 [V, d]");
  c10::cuda::CUDAGuard guard(dy.device());
  auto flat = ids.reshape({-1}).contiguous();
  auto dy2 = dy.reshape({flat.numel(), dw.size(1)}).contiguous();
  const int64_t seg = std::min<int64_t>(flat.numel(), embedding_sort_segment());
  auto keys = torch::empty({std::max<int64_t>(seg, 1)}, flat.options());  // uint64 keys in int64 storage
  embedding_bwd(flat.data_ptr<int64_t>(), dy2.data_ptr(), dw.data_ptr<float>(),
                reinterpret_cast<uint64_t*>(keys.data_ptr<int64_t>()), int(flat.numel()), int(dw.size(1)), start,
                dw.size(0), cur_stream());
}

// ---- cross-entropy --------------------------------------------------------------------

torch::Tensor xent_stats_t(torch::Tensor logits, torch::Tensor labels, int64_t start) {
  check_cuda_bf16(logits, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be 2-D");
  TORCH_CHECK(labels.scalar_type() == torch::kLong && labels.numel() == logits.size(0) && labels.is_contiguous(),
              "labels must be int64 [rows]");
  c10::cuda::CUDAGuard guard(logits.device());
  auto stats = torch::empty({logits.size(0), 3}, logits.options().dtype(torch::kFloat));
  xent_stats(logits.data_ptr(), logits.stride(0), labels.data_ptr<int64_t>(), stats.data_ptr<float>(),
             int(logits.size(0)), int(logits.size(1)), start, cur_stream());
  return stats;
}

void xent_grad_t(torch::Tensor logits, torch::Tensor labels, torch::Tensor lse, torch::Tensor scale, int64_t start) {
  check_cuda_bf16(logits, "logits");
  TORCH_CHECK(lse.scalar_type() == torch::kFloat && lse.numel() == logits.size(0) && lse.is_contiguous(), "lse");
  TORCH_CHECK(scale.scalar_type() == torch::kFloat && scale.numel() == 1 && scale.is_cuda(), "scale must be a CUDA fp32 scalar");
  c10::cuda::CUDAGuard guard(logits.device());
  xent_grad(logits.data_ptr(), logits.stride(0), labels.data_ptr<int64_t>(), lse.data_ptr<float>(),
            scale.data_ptr<float>(), int(logits.size(0)), int(logits.size(1)), start, cur_stream());
}

// ---- attention ------------------------------------------------------------------------

std::vector<torch::Tensor> attn_fwd_t(torch::Tensor qkv, int64_t seq, int64_t hq, int64_t hkv, int64_t d, double scale) {
  check_cuda_bf16(qkv, "qkv");
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.size(1) == (hq + 2 * hkv) * d, "qkv must be [T, (hq+2hkv)*d]");
  c10::cuda::CUDAGuard guard(qkv.device());
  const int64_t rows = qkv.size(0);
  auto out = torch::empty({rows, hq * d}, qkv.options());
  auto lse = torch::empty({rows / seq, hq, seq}, qkv.options().dtype(torch::kFloat));
  attn_fwd(qkv.data_ptr(), qkv.stride(0), out.data_ptr(), out.stride(0), lse.data_ptr<float>(), int(rows), int(seq),
           int(hq), int(hkv), int(d), float(scale), error_word(qkv.device()), cur_stream());
  return {out, lse};
}

torch::Tensor attn_bwd_t(torch::Tensor qkv, torch::Tensor out, torch::Tensor dout, torch::Tensor lse, int64_t seq,
                         int64_t hq, int64_t hkv, int64_t d, double scale) {
  check_cuda_bf16(qkv, "qkv");
  check_cuda_bf16(out, "out");
  check_cuda_bf16(dout, "dout");
  TORCH_CHECK(dout.stride(1) == 1 && out.stride(1) == 1, "attention tensors need unit inner stride");
  c10::cuda::CUDAGuard guard(qkv.device());
  const int64_t rows = qkv.size(0);
  auto dqkv = torch::empty({rows, (hq + 2 * hkv) * d}, qkv.options());
  auto delta = torch::empty_like(lse);
  attn_bwd(qkv.data_ptr(), qkv.stride(0), out.data_ptr(), out.stride(0), dout.data_ptr(), dout.stride(0),
           lse.data_ptr<float>(), delta.data_ptr<float>(), dqkv.data_ptr(), dqkv.stride(0), int(rows), int(seq),
           int(hq), int(hkv), int(d), float(scale), error_word(qkv.device()), cur_stream());
  return dqkv;
}


// ---- debugging aid: native backtrace on SIGSEGV ---------------------------------------

static void crash_handler(int sig) {
  void* frames[64];
  const int n = backtrace(frames, 64);
  const char msg[] = "\n[resihp] native backtrace:\n";
  (void)!write(2, msg, sizeof(msg) - 1);
  backtrace_symbols_fd(frames, n, 2);
  signal(sig, SIG_DFL);
  raise(sig);
}

void install_crash_handler() { signal(SIGSEGV, crash_handler); }

// ---- symmetric workspace + fused TP collectives ---------------------------------------

template <class T>
static T* as_ptr(int64_t v) { return reinterpret_cast<T*>(static_cast<uintptr_t>(v)); }

py::tuple symm_alloc_t(int64_t bytes) {
  cudaIpcMemHandle_t h;
  void* p = symm_alloc(bytes, &h);
  return py::make_tuple(reinterpret_cast<int64_t>(p), py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)));
}

int64_t symm_open_t(py::bytes handle) {
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  return reinterpret_cast<int64_t>(symm_open(s.data()));
}

void symm_close_t(int64_t p) { symm_close(as_ptr<void>(p)); }

// Debug helpers for guard bytes around workspace buffers (synchronous, any device memory).
void debug_fill_bytes_t(int64_t p, int64_t bytes, int64_t value) {
  C10_CUDA_CHECK(cudaMemset(as_ptr<void>(p), int(value & 0xff), size_t(bytes)));
}

py::bytes debug_read_bytes_t(int64_t p, int64_t bytes) {
  std::string out(size_t(bytes), '\0');
  C10_CUDA_CHECK(cudaMemcpy(out.data(), as_ptr<const void>(p), size_t(bytes), cudaMemcpyDeviceToHost));
  return py::bytes(out);
}
void symm_free_t(int64_t p) { symm_free(as_ptr<void>(p)); }

int64_t fused_grid_t(int64_t m, int64_t n, int64_t tp) { return fused_grid(int(m), int(n), int(tp)); }
int64_t fused_slices_t(int64_t rows_per_rank) { return fused_slices(int(rows_per_rank)); }
int64_t fused_tile_claims_t(int64_t t_rows, int64_t n, int64_t grid) {
  return fused_tile_claims(int(t_rows), int(n), int(grid));
}
int64_t fused_copy_claims_t(int64_t mode, int64_t t_rows, int64_t n, int64_t tp, int64_t slices, int64_t xg_chunks,
                            int64_t grid) {
  return fused_copy_claims(int(mode), int(t_rows), int(n), int(tp), int(slices), int(xg_chunks), int(grid));
}

// The peers of one fused call as a flat int64 list: rank, tp, rows_per_rank, slices, epoch,
// ar_epoch, tile_ctr, tile_base, copy_ctr, copy_base, then tp addresses each of land,
// ag_cnt, recv, rs_cnt, out_land, ar_cnt (0 where a call does not use them).
static FusedPeers decode_peers(const std::vector<int64_t>& v) {
  TORCH_CHECK(v.size() >= 10, "fused peers: header missing");
  FusedPeers p{};
  p.rank = int(v[0]);
  p.tp = int(v[1]);
  p.rows_per_rank = int(v[2]);
  p.slices = int(v[3]);
  p.epoch = unsigned(v[4]);
  p.ar_epoch = unsigned(v[5]);
  p.tile_ctr = as_ptr<unsigned>(v[6]);
  p.tile_base = unsigned(v[7]);
  p.copy_ctr = as_ptr<unsigned>(v[8]);
  p.copy_base = unsigned(v[9]);
  TORCH_CHECK(p.tp >= 2 && p.tp <= kFusedMaxTp && v.size() == size_t(10 + 6 * p.tp + 3), "fused peers: bad length");
  for (int r = 0; r < p.tp; ++r) {
    p.land[r] = as_ptr<__nv_bfloat16>(v[10 + r]);
    p.ag_cnt[r] = as_ptr<unsigned>(v[10 + p.tp + r]);
    p.recv[r] = as_ptr<__nv_bfloat16>(v[10 + 2 * p.tp + r]);
    p.rs_cnt[r] = as_ptr<unsigned>(v[10 + 3 * p.tp + r]);
    p.out_land[r] = as_ptr<__nv_bfloat16>(v[10 + 4 * p.tp + r]);
    p.ar_cnt[r] = as_ptr<unsigned>(v[10 + 5 * p.tp + r]);
  }
  p.send = as_ptr<__nv_bfloat16>(v[10 + 6 * p.tp]);
  p.send_cnt = as_ptr<unsigned>(v[11 + 6 * p.tp]);
  p.own_cnt = as_ptr<unsigned>(v[12 + 6 * p.tp]);
  return p;
}

void ag_gemm_t(torch::Tensor x_local, c10::optional<torch::Tensor> xg, torch::Tensor w, bool w_mn, torch::Tensor y,
               std::vector<int64_t> peers, int64_t grid) {
  check_cuda_bf16(x_local, "x_local");
  check_cuda_bf16(w, "w");
  check_cuda_bf16(y, "y");
  const FusedPeers p = decode_peers(peers);
  TORCH_CHECK(x_local.is_contiguous() && y.is_contiguous() && w.stride(1) == 1, "fused AG-GEMM tensors must be contiguous");
  const int64_t k = x_local.size(1);
  const int64_t t = x_local.size(0) * p.tp;
  const int64_t n = y.size(1);
  TORCH_CHECK(y.size(0) == t, "fused AG-GEMM shapes");
  void* xg_ptr = nullptr;
  if (xg.has_value()) {
    check_cuda_bf16(*xg, "xg");
    TORCH_CHECK(xg->is_contiguous() && xg->size(0) == t && xg->size(1) == k, "fused AG-GEMM gathered-copy shape");
    xg_ptr = xg->data_ptr();
  }
  TORCH_CHECK(w_mn ? (w.size(0) == k && w.size(1) == n) : (w.size(0) == n && w.size(1) == k), "fused AG-GEMM weight");
  c10::cuda::CUDAGuard guard(x_local.device());
  fused_ag_gemm(x_local.data_ptr(), xg_ptr, w.data_ptr(), w.stride(0), w_mn, y.data_ptr(), y.stride(0), int(t),
                int(n), int(k), p, int(grid), error_word(x_local.device()), cur_stream());
}

// RS (all_reduce false): y is this rank's [T/tp, N] rows; AR: y is the full [T, N].
void gemm_rs_t(torch::Tensor h, torch::Tensor w, bool w_mn, torch::Tensor y, bool all_reduce,
               std::vector<int64_t> peers, int64_t grid) {
  check_cuda_bf16(h, "h");
  check_cuda_bf16(w, "w");
  check_cuda_bf16(y, "y");
  const FusedPeers p = decode_peers(peers);
  TORCH_CHECK(h.is_contiguous() && y.is_contiguous() && w.stride(1) == 1, "fused GEMM-RS tensors must be contiguous");
  const int64_t t = h.size(0), k = h.size(1), n = y.size(1);
  TORCH_CHECK(all_reduce ? y.size(0) == t : y.size(0) * p.tp == t, "fused GEMM-RS/AR shapes");
  TORCH_CHECK(w_mn ? (w.size(0) == k && w.size(1) == n) : (w.size(0) == n && w.size(1) == k), "fused GEMM-RS weight");
  c10::cuda::CUDAGuard guard(h.device());
  fused_gemm_rs(h.data_ptr(), w.data_ptr(), w.stride(0), w_mn, y.data_ptr(), y.stride(0), int(t), int(n), int(k),
                all_reduce, p, int(grid), error_word(h.device()), cur_stream());
}

// ---- flat-state regions and the peer-state kernels ----------------------------------------

// A zeroed, IPC-exported device allocation wrapped as a uint8 tensor. The memory is
// released when the last tensor viewing it dies (the deleter frees it on its device).
py::tuple symm_region_t(int64_t bytes, int64_t device) {
  TORCH_CHECK(bytes > 0, "region size must be positive");
  c10::cuda::CUDAGuard guard(c10::Device(c10::kCUDA, device));
  cudaIpcMemHandle_t h;
  void* p = symm_alloc(bytes, &h);
  const int dev = int(device);
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  auto t = torch::from_blob(
      p, {bytes},
      [dev](void* q) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(dev);
        cudaFree(q);
        cudaSetDevice(prev);
      },
      opts);
  return py::make_tuple(t, py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)));
}

int64_t dp_grid_t(int64_t n, int64_t device) {
  return dp_grid(n, at::cuda::getDeviceProperties(device)->multiProcessorCount);
}

void dp_allreduce_adamw_t(std::vector<int64_t> grads, int64_t me, torch::Tensor sum_out, torch::Tensor p,
                          torch::Tensor m, torch::Tensor v, c10::optional<torch::Tensor> p_bf16, double lr, double b1,
                          double b2, double eps, double wd, int64_t step, double grad_scale, int64_t flags_local,
                          std::vector<int64_t> flags_peer, int64_t epoch, int64_t grid,
                          std::vector<int64_t> sums_peer, int64_t flags2_local, std::vector<int64_t> flags2_peer) {
  for (auto* t : {&sum_out, &p, &m, &v})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat && t->is_contiguous() && t->numel() == p.numel(),
                "DP AdamW buffers must be contiguous fp32 of equal size");
  const int64_t dp = int64_t(grads.size());
  TORCH_CHECK(dp >= 1 && dp <= kMaxDp && int64_t(flags_peer.size()) == dp && me >= 0 && me < dp,
              "one gradient buffer and one flag array per DP rank");
  void* pb = nullptr;
  if (p_bf16.has_value()) {
    TORCH_CHECK(p_bf16->scalar_type() == torch::kBFloat16 && p_bf16->numel() == p.numel() && p_bf16->is_contiguous(),
                "bf16 copy must match");
    pb = p_bf16->data_ptr();
  }
  c10::cuda::CUDAGuard guard(p.device());
  std::vector<const float*> g;
  std::vector<unsigned*> f;
  for (auto x : grads) g.push_back(as_ptr<const float>(x));
  for (auto x : flags_peer) f.push_back(as_ptr<unsigned>(x));
  const AdamWCoef c = adamw_coef(float(lr), float(b1), float(b2), float(eps), float(wd), step, float(grad_scale));
  const bool push = !sums_peer.empty();
  TORCH_CHECK(!push || (int64_t(sums_peer.size()) == dp && int64_t(flags2_peer.size()) == dp && flags2_local != 0),
              "the push variant needs one receiving buffer and one second flag array per DP rank");
  std::vector<float*> sp;
  std::vector<unsigned*> f2;
  for (auto x : sums_peer) sp.push_back(as_ptr<float>(x));
  for (auto x : flags2_peer) f2.push_back(as_ptr<unsigned>(x));
  dp_allreduce_adamw(g.data(), int(dp), int(me), sum_out.data_ptr<float>(), p.data_ptr<float>(), m.data_ptr<float>(),
                     v.data_ptr<float>(), pb, p.numel(), c, as_ptr<unsigned>(flags_local), f.data(), unsigned(epoch),
                     int(grid), error_word(p.device()), cur_stream(), push ? sp.data() : nullptr,
                     push ? as_ptr<unsigned>(flags2_local) : nullptr, push ? f2.data() : nullptr);
}

// descs: int64 [n, 9] on the device, one CopyDesc per row (see launch.h for the fields).
void reshard_gather_t(torch::Tensor descs, int64_t items) {
  static_assert(sizeof(CopyDesc) == 9 * sizeof(int64_t), "CopyDesc is nine 8-byte fields");
  TORCH_CHECK(descs.is_cuda() && descs.scalar_type() == torch::kLong && descs.is_contiguous() && descs.dim() == 2 &&
                  descs.size(1) == 9, "copy descriptors must be a contiguous int64 [n, 9] CUDA tensor");
  c10::cuda::CUDAGuard guard(descs.device());
  reshard_gather(reinterpret_cast<const CopyDesc*>(descs.data_ptr<int64_t>()), int(descs.size(0)), items,
                 error_word(descs.device()), at::cuda::getDeviceProperties(descs.device().index())->multiProcessorCount,
                 cur_stream());
}

}  // namespace resihp

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "resihp sm_100a kernels";
  m.def("read_and_clear_error", &resihp::read_and_clear_error, "synchronising read+reset of the kernel error word");
  m.def("peer_wait_budget_ns", [] { return int64_t(resihp::peer_wait_budget_ns()); },
        "budget of each in-kernel wait on another GPU's flag (ns)");
  m.def("set_peer_wait_budget_ns", [](int64_t ns) { resihp::set_peer_wait_budget_ns(uint64_t(ns)); },
        "set the budget of each in-kernel wait on another GPU's flag (ns)");
  m.def("fused_red_slices", &resihp::fused_red_slices, "row slices per own tile of the fused RS / AR reduction");
  m.def("set_fused_trace", [](int64_t ptr) { resihp::set_fused_trace(reinterpret_cast<uint64_t*>(ptr)); },
        "profiling aid: per-CTA timer stamps of the fused TP kernels into a device buffer (0: off)");
  m.def("fused_trace_slots", &resihp::fused_trace_slots, "stamps per CTA of the fused-kernel trace");
  m.def("set_fused_push_depth", &resihp::set_fused_push_depth,
        "RS / AR partial-tile pushes in flight per copy thread: 2 pipelined, 1 one at a time (default)");
  m.def("gemm", &resihp::gemm, "tcgen05 bf16 GEMM", py::arg("a"), py::arg("a_mn"), py::arg("b"), py::arg("b_mn"),
        py::arg("c"), py::arg("epi"), py::arg("alpha") = 1.0, py::arg("residual") = py::none(),
        py::arg("max_ctas") = 0, py::arg("force_bn") = 0);
  m.def("rmsnorm_fwd", &resihp::rmsnorm_fwd_t);
  m.def("rmsnorm_bwd", &resihp::rmsnorm_bwd_t);
  m.def("rope", &resihp::rope_t);
  m.def("swiglu_fwd", &resihp::swiglu_fwd_t);
  m.def("swiglu_bwd", &resihp::swiglu_bwd_t);
  m.def("adamw", &resihp::adamw_t);
  m.def("embedding_fwd", &resihp::embedding_fwd_t);
  m.def("embedding_bwd", &resihp::embedding_bwd_t);
  m.def("xent_stats", &resihp::xent_stats_t);
  m.def("xent_grad", &resihp::xent_grad_t);
  m.def("attn_fwd", &resihp::attn_fwd_t);
  m.def("attn_bwd", &resihp::attn_bwd_t);
  m.def("install_crash_handler", &resihp::install_crash_handler);
  m.def("symm_alloc", &resihp::symm_alloc_t);
  m.def("symm_open", &resihp::symm_open_t);
  m.def("symm_close", &resihp::symm_close_t);
  m.def("symm_free", &resihp::symm_free_t);
  m.def("debug_fill_bytes", &resihp::debug_fill_bytes_t);
  m.def("debug_read_bytes", &resihp::debug_read_bytes_t);
  m.def("fused_grid", &resihp::fused_grid_t);
  m.def("fused_slices", &resihp::fused_slices_t);
  m.def("fused_tile_claims", &resihp::fused_tile_claims_t);
  m.def("fused_copy_claims", &resihp::fused_copy_claims_t);
  m.def("ag_gemm", &resihp::ag_gemm_t, py::arg("x_local"), py::arg("xg"), py::arg("w"), py::arg("w_mn"), py::arg("y"),
        py::arg("peers"), py::arg("grid"));
  m.def("gemm_rs", &resihp::gemm_rs_t, py::arg("h"), py::arg("w"), py::arg("w_mn"), py::arg("y"),
        py::arg("all_reduce"), py::arg("peers"), py::arg("grid"));
  m.def("symm_region", &resihp::symm_region_t);
  m.def("dp_grid", &resihp::dp_grid_t);
  m.def("dp_allreduce_adamw", &resihp::dp_allreduce_adamw_t, py::arg("grads"), py::arg("me"), py::arg("sum_out"),
        py::arg("p"), py::arg("m"), py::arg("v"), py::arg("p_bf16"), py::arg("lr"), py::arg("b1"), py::arg("b2"),
        py::arg("eps"), py::arg("wd"), py::arg("step"), py::arg("grad_scale"), py::arg("flags_local"),
        py::arg("flags_peer"), py::arg("epoch"), py::arg("grid"), py::arg("sums_peer") = std::vector<int64_t>{},
        py::arg("flags2_local") = 0, py::arg("flags2_peer") = std::vector<int64_t>{});
  m.def("reshard_gather", &resihp::reshard_gather_t);
}
