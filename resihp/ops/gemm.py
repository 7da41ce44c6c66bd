"""Linear-layer products on the tcgen05 GEMM (``csrc/gemm.cu``).

All three products of a bias-free linear layer ``y = x w^T`` read their operands in
place (no transposes): the kernel takes each operand K-major or MN-major. (Reference:
``F.linear`` at ``resihp/parallel/tp.py:235-248,272`` and its autograd products.)

bf16 CUDA tensors always run the hand-written kernel; FP32 tensors (CPU or CUDA)
compute in plain torch, the FP32 reference path.
"""

from __future__ import annotations

import os

import torch

from . import _ext

EPI_BF16 = 0
EPI_F32 = 1
EPI_ACC_F32 = 2
EPI_ADD_BF16 = 3
EPI_RED_F32 = 4

#: Weight-gradient accumulation through ``red.global.add`` (no load in the epilogue)
#: instead of load-add-store; same sums except that subnormals flush to zero. Each
#: element receives exactly one addition per launch, so the result is deterministic.
#: Measured 14-25 % faster on the 1.3B weight-gradient shapes (``bench_kernels.py
#: gemm_time``); ``RESIHP_WGRAD_RED=0`` selects load-add-store.
WGRAD_RED = os.environ.get("RESIHP_WGRAD_RED", "1") == "1"


def _cuda(*tensors) -> bool:
    return tensors[0].is_cuda and tensors[0].dtype == torch.bfloat16


def linear(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w.T`` (+ ``residual``), x: [..., K], w: [N, K]."""
    if not _cuda(x):
        y = torch.nn.functional.linear(x, w)
        return y if residual is None else y + residual
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    out = torch.empty((x2.shape[0], w.shape[0]), dtype=torch.bfloat16, device=x.device)
    if residual is None:
        _ext.require().gemm(x2, False, w, False, out, EPI_BF16)
    else:
        r2 = residual.reshape(-1, w.shape[0])
        _ext.require().gemm(x2, False, w, False, out, EPI_ADD_BF16, 1.0, r2)
    return out.view(*lead, w.shape[0])


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``dy @ w``: the input gradient of ``x @ w.T``; dy: [..., N], w: [N, K]."""
    if not _cuda(dy):
        return dy @ w
    lead = dy.shape[:-1]
    d2 = dy.reshape(-1, dy.shape[-1])
    out = torch.empty((d2.shape[0], w.shape[1]), dtype=torch.bfloat16, device=dy.device)
    _ext.require().gemm(d2, False, w, True, out, EPI_BF16)
    return out.view(*lead, w.shape[1])


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """``dy^T @ x`` in FP32: the weight gradient of ``x @ w.T``.

    With ``accumulate`` the product is added into ``out`` (an FP32 main-grad buffer),
    which is how gradients of successive micro-batches accumulate without a separate
    add kernel.
    """
    d2 = dy.reshape(-1, dy.shape[-1])
    x2 = x.reshape(-1, x.shape[-1])
    if not _cuda(dy):
        g = d2.t().float() @ x2.float()
        if out is None:
            return g
        if accumulate:
            out.add_(g)
        else:
            out.copy_(g)
        return out
    if out is None:
        out = torch.empty((d2.shape[1], x2.shape[1]), dtype=torch.float32, device=dy.device)
        accumulate = False
    _ext.require().gemm(d2, True, x2, True, out, ((EPI_RED_F32 if WGRAD_RED else EPI_ACC_F32) if accumulate
                                                 else EPI_F32))
    return out


#: Codes a kernel records in its device's error word (``ErrorCode`` in csrc/common.cuh).
ERROR_CODES = {
    1: "TMA producer waited past its budget for a free shared-memory stage",
    2: "MMA issuer waited past its budget for a filled stage or a free accumulator",
    3: "epilogue waited past its budget for a finished accumulator",
    4: "a wait on another GPU's flag ran out its budget (peer never arrived)",
    5: "a bounds check of the checked build skipped an access",
}
PEER_WAIT = 4


class KernelError(RuntimeError):
    """A kernel reported an error code (a bounded wait that ran out, a failed bounds
    check) instead of hanging or faulting; ``code`` is the recorded code."""

    def __init__(self, code: int, device_index: int):
        self.code = int(code)
        self.device_index = int(device_index)
        what = ERROR_CODES.get(self.code, "unknown error code")
        super().__init__(f"resihp kernel reported error code {self.code} on cuda:{self.device_index}: {what}")


def check_device_errors(device: torch.device | int | None = None) -> None:
    """Raise :class:`KernelError` if any kernel on ``device`` reported a timed-out wait
    or a bounds error since the last check (the word is cleared by the read)."""
    if not torch.cuda.is_available():
        return
    index = torch.cuda.current_device() if device is None else torch.device("cuda", device).index if isinstance(device, int) else (device.index or 0)
    code = _ext.require().read_and_clear_error(index)
    if code:
        raise KernelError(code, index)
