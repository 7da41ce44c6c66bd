"""The allocation-free RMSNorm-backward entry point, called through its exported C symbol.

Some callers of this library cannot allocate device memory (a host program without a
device allocator of its own, or a runtime that reserved all device memory up front):
``resihp_rmsnorm_bwd_noalloc`` takes only the caller's inputs and outputs and keeps its
scratch in a fixed device array inside the library. This test checks it against the
allocating entry point on two calls in a row (the second call reuses the scratch the
first one left behind). It is collected last on purpose.
"""

import ctypes

import pytest
import torch

from resihp.ops import _ext

pytestmark = pytest.mark.gpu


def _lib():
    lib = ctypes.CDLL(_ext.library_path())
    fn = lib.resihp_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    lib.resihp_noalloc_strerror.restype = ctypes.c_char_p
    lib.resihp_noalloc_strerror.argtypes = [ctypes.c_int]
    return lib


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _inputs(rows, d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    dy = torch.randn(rows, d, device="cuda", generator=g).bfloat16()
    s = torch.randn(rows, d, device="cuda", generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    rstd = torch.rsqrt(s.float().pow(2).mean(-1) + 1e-5).contiguous()
    dres = torch.randn(rows, d, device="cuda", generator=g).bfloat16()
    return dy, s, w, rstd, dres


@pytest.mark.parametrize("rows,d,with_res", [(333, 2048, True), (1000, 256, False), (64, 5120, True)])
def test_noalloc_matches_allocating_entry_point(rows, d, with_res):
    lib = _lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        dy, s, w, rstd, dres = _inputs(rows, d, seed=17 * call + d)
        dres = dres if with_res else None
        start = torch.randn(d, device="cuda")
        dw_ref = start.clone()
        ds_ref = _ext.require().rmsnorm_bwd(dy, s, w, rstd, dres, dw_ref, True)
        dw = start.clone()
        ds = torch.empty_like(dy)
        code = lib.resihp_rmsnorm_bwd_noalloc(
            _ptr(dy), _ptr(s), _ptr(w), _ptr(rstd), _ptr(dres), _ptr(ds), _ptr(dw), 1, rows, d, stream
        )
        assert code == 0, lib.resihp_noalloc_strerror(code)
        torch.cuda.synchronize()
        assert torch.allclose(ds.float(), ds_ref.float(), rtol=1e-2, atol=1e-2)
        assert torch.allclose(dw, dw_ref, rtol=1e-5, atol=1e-5)


def test_noalloc_rejects_bad_sizes():
    lib = _lib()
    dy, s, w, rstd, _ = _inputs(8, 256, seed=1)
    ds = torch.empty_like(dy)
    dw = torch.zeros(256, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    code = lib.resihp_rmsnorm_bwd_noalloc(_ptr(dy), _ptr(s), _ptr(w), _ptr(rstd), None, _ptr(ds), _ptr(dw), 0, 8, 100, stream)
    assert code == 1 and b"unsupported width" in lib.resihp_noalloc_strerror(code)


def test_noalloc_leaves_an_earlier_error_to_its_owner():
    """A CUDA error pending from an unrelated earlier call (here a host-side one: an
    invalid device ordinal) is neither reported as this entry point's failure nor
    cleared: the call returns the pending-error code and launches nothing."""
    lib = _lib()
    cudart = ctypes.CDLL("libcudart.so.12")  # the runtime instance the extension uses
    cudart.cudaSetDevice.argtypes = [ctypes.c_int]
    cudart.cudaSetDevice.restype = ctypes.c_int
    cudart.cudaGetLastError.restype = ctypes.c_int
    dy, s, w, rstd, _ = _inputs(8, 256, seed=2)
    ds = torch.zeros_like(dy)
    dw = torch.zeros(256, device="cuda")
    torch.cuda.synchronize()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert cudart.cudaSetDevice(1 << 20) != 0  # leaves cudaErrorInvalidDevice pending
    code = lib.resihp_rmsnorm_bwd_noalloc(_ptr(dy), _ptr(s), _ptr(w), _ptr(rstd), None, _ptr(ds), _ptr(dw), 0, 8, 256,
                                          stream)
    pending = cudart.cudaGetLastError()  # still there for its owner, then cleared
    assert code == 4 and b"pending" in lib.resihp_noalloc_strerror(code)
    assert pending != 0 and cudart.cudaGetLastError() == 0
    torch.cuda.synchronize()
    assert torch.count_nonzero(ds) == 0 and torch.count_nonzero(dw) == 0  # nothing ran
