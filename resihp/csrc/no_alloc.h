// Allocation-free C entry point of the RMSNorm backward pass.
//
// This entry point has no counterpart in the reference implementation: it exists for
// callers of this library that cannot allocate device memory themselves -- a C, C++ or
// Fortran host program that links the library without a device allocator of its own,
// or a runtime that reserves all device memory at start-up and forbids later
// cudaMalloc calls (cudaMalloc can synchronise the device, and it can fail once
// memory is fragmented or fully reserved). Such a caller passes only its own inputs
// and outputs; the kernel's scratch lives in a fixed-size device array compiled into
// the library.
//
// Limits and contract (see norm.cu for the implementation):
//   * Scratch: RESIHP_NOALLOC_SCRATCH_FLOATS fp32 values (16 MiB) per GPU that loads
//     the library, held until the process exits. A call whose scratch need
//     (row slots x width, the same launch shape as the allocating entry point) is
//     larger is rejected with RESIHP_NOALLOC_TOO_LARGE before anything is launched.
//   * Set-up: the first call on a device looks up the device address of the scratch
//     array for that device (cudaGetSymbolAddress, with that device current) and keeps
//     it for later calls. Make that first call before any stream capture. A reset of the
//     device's primary context (cudaDeviceReset) unmaps the array and so invalidates
//     the kept address: call resihp_noalloc_forget_device() for that device after such
//     a reset, and the next call looks the address up again.
//   * Errors: a CUDA error already pending on the calling thread when the call starts
//     is not attributed to this call; the call returns RESIHP_NOALLOC_PENDING_ERROR,
//     launches nothing and leaves that error in place for its owner to read.
//   * Sharing: every call on a device uses the same scratch array, and each call
//     overwrites the whole part of it that it reads, so nothing has to be cleared in
//     between. Calls whose work overlaps on the GPU (different streams without ordering
//     between them) race on the scratch array and give wrong results: order them.
//   * No allocation: the entry point calls no cudaMalloc, cudaFree or any allocating
//     library routine (torch's included).
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RESIHP_NOALLOC_SCRATCH_FLOATS (4 * 1024 * 1024)

enum {
  RESIHP_NOALLOC_OK = 0,
  RESIHP_NOALLOC_BAD_ARGUMENT = 1,  // null pointer, rows < 1, or an unsupported width
  RESIHP_NOALLOC_TOO_LARGE = 2,     // the scratch need exceeds RESIHP_NOALLOC_SCRATCH_FLOATS
  RESIHP_NOALLOC_CUDA_ERROR = 3,    // a CUDA runtime call or a launch of this call failed
  RESIHP_NOALLOC_PENDING_ERROR = 4, // an earlier CUDA error was pending; nothing was launched
};

// Backward of y = rmsnorm(s) * w over bf16 rows of width d (see norm.cu):
//   ds = rstd * (dy*w - s_hat * mean(dy*w*s_hat)) (+ dres, if dres is not null)
//   dw = (dw if accumulate else 0) + sum over rows of dy * s_hat     (fp32)
// dy, s, dres, ds: [rows, d] bf16 row-major; w: [d] bf16; rstd: [rows] fp32;
// dw: [d] fp32. All pointers are device pointers owned by the caller. The work is
// enqueued on `stream`; the return code reports argument and launch errors.
int resihp_rmsnorm_bwd_noalloc(const void* dy, const void* s, const void* w, const float* rstd, const void* dres,
                               void* ds, float* dw, int accumulate, int rows, int d, cudaStream_t stream);

// Drop the kept scratch address of `device` (after a reset of its primary context).
void resihp_noalloc_forget_device(int device);

// Human-readable text for a return code of the entry point above.
const char* resihp_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif
