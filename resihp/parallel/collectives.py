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


def copy_to_tp(x, group):
    return x if tp_size(group) == 1 else _Copy.apply(x, group)


def reduce_from_tp(x, group):
    return x if tp_size(group) == 1 else _Reduce.apply(x, group)


def gather_tokens(x, group):
    return x if tp_size(group) == 1 else _GatherTokens.apply(x, group)


def scatter_tokens(x, group):
    return x if tp_size(group) == 1 else _ScatterTokens.apply(x, group)
