"""Tensor-parallel communication as autograd functions (Megatron f / g and SP forms).

* ``copy_to_tp``      (f): identity forward, all-reduce of the input gradient backward;
* ``reduce_from_tp``  (g): all-reduce forward, identity backward;
* ``gather_tokens``   (SP): all-gather along tokens forward, reduce-scatter backward;
* ``scatter_tokens``  (SP): reduce-scatter along tokens forward, all-gather backward.

Reference: ``resihp/parallel/tp.py:63-110`` (f, g and the logit gather; the logit
gather has no counterpart here because the loss is vocab-parallel). All four are
no-ops at TP degree 1. The fused GEMM+collective kernels in
:mod:`resihp.parallel.fused` replace the SP pair on the B200 hot path.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch.autograd import Function


def tp_size(group) -> int:
    return 1 if group is None else dist.get_world_size(group)


class _Copy(Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, grad):
        grad = grad.contiguous().clone()
        dist.all_reduce(grad, group=ctx.group)
        return grad, None


class _Reduce(Function):
    @staticmethod
    def forward(ctx, x, group):
        x = x.contiguous().clone()
        dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, grad):
        return grad, None


def _all_gather_rows(x, group):
    n = dist.get_world_size(group)
    out = torch.empty((x.shape[0] * n,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def _reduce_scatter_rows(x, group):
    n = dist.get_world_size(group)
    out = torch.empty((x.shape[0] // n,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
    return out


class _GatherTokens(Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _all_gather_rows(x, group)

    @staticmethod
    def backward(ctx, grad):
        return _reduce_scatter_rows(grad, ctx.group), None


class _ScatterTokens(Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _reduce_scatter_rows(x, group)

    @staticmethod
    def backward(ctx, grad):
        return _all_gather_rows(grad, ctx.group), None


class _ColumnParallelLinear(Function):
    """``gather_tokens(h) @ w.T`` (SP) or ``copy_to_tp(h) @ w.T``, with the backward's
    input-gradient collective overlapped with the weight-gradient product.

    Megatron's order: the input gradient is computed first and its reduce-scatter (SP)
    or all-reduce is started asynchronously; the weight gradient -- which needs no
    communication -- runs while it is in flight; the collective is awaited last. The
    sums are the same as with the collective after both products.
    """

    @staticmethod
    def forward(ctx, h, w, main_grad, group, sp):
        from ..ops import functional as fn

        x = _all_gather_rows(h, group) if sp else h
        ctx.save_for_backward(x, w)
        ctx.main_grad, ctx.group, ctx.sp = main_grad, group, sp
        ctx.kernel = fn.on_kernels(x)
        return fn.linear(x, w) if not ctx.kernel else _kernel_linear(x, w)

    @staticmethod
    def backward(ctx, dy):
        from ..ops.gemm import linear_dgrad, linear_wgrad

        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = linear_dgrad(dy, w)
        n = dist.get_world_size(ctx.group)
        if ctx.sp:
            out = torch.empty((dx.shape[0] // n,) + tuple(dx.shape[1:]), dtype=dx.dtype, device=dx.device)
            work = dist.reduce_scatter_tensor(out, dx.contiguous(), group=ctx.group, async_op=True)
        else:
            out = dx.contiguous()
            work = dist.all_reduce(out, group=ctx.group, async_op=True)
        dw = None
        if ctx.kernel:
            if ctx.main_grad is not None:
                linear_wgrad(dy, x, out=ctx.main_grad, accumulate=True)
        elif ctx.needs_input_grad[1]:
            dw = linear_wgrad(dy, x).to(w.dtype)
        work.wait()
        return out, dw, None, None, None


def _kernel_linear(x, w):
    from ..ops.gemm import linear

    return linear(x, w)


def column_parallel_linear(h, w, main_grad, group, sp: bool):
    """The column-parallel linear of a TP group of two or more (see :class:`_ColumnParallelLinear`)."""
    return _ColumnParallelLinear.apply(h, w, main_grad, group, sp)


def copy_to_tp(x, group):
    return x if tp_size(group) == 1 else _Copy.apply(x, group)


def reduce_from_tp(x, group):
    return x if tp_size(group) == 1 else _Reduce.apply(x, group)


def gather_tokens(x, group):
    return x if tp_size(group) == 1 else _GatherTokens.apply(x, group)


def scatter_tokens(x, group):
    return x if tp_size(group) == 1 else _ScatterTokens.apply(x, group)
