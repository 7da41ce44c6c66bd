"""Fused sequence-parallel TP linears over NVLink peer memory (csrc/fused_gemm.cu).

* :func:`ag_linear`  -- column-parallel: ``y = all_gather_tokens(x_r) @ w.T`` as one
  AG->GEMM kernel; backward: the input gradient is one GEMM->RS kernel and the weight
  gradient reuses the gathered input the forward kernel left in its gather buffer.
* :func:`linear_rs`  -- row-parallel: ``y_r = reduce_scatter_tokens(h @ w.T)`` as one
  GEMM->RS kernel; backward: the input gradient is one AG->GEMM kernel over the output
  gradient, whose gathered copy feeds the weight gradient.

Both replace the NCCL pair ``gather_tokens`` / ``scatter_tokens`` of
:mod:`resihp.parallel.collectives` (the baseline). They exchange data through a
:class:`SymmetricWorkspace` per TP group: one CUDA-IPC-shared region per rank holding
the cross-GPU flags and counters, two publish slots for the AG input and two receive
slots per source for the RS partials. Nothing in the workspace is multicast.

All ranks of a TP group issue their fused calls in the same order (they follow the same
model code), which is what the epoch counters rely on.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist
from torch.autograd import Function

from ..ops import _ext
from ..ops.gemm import linear_wgrad

ENABLED = os.environ.get("RESIHP_FUSED_TP", "1") != "0"
DEBUG = os.environ.get("RESIHP_FUSED_DEBUG", "0") == "1"


def _debug_check(what: str, device) -> None:
    """Debug builds: synchronise after a fused launch and surface its error word."""
    if not DEBUG:
        return
    import sys

    torch.cuda.synchronize(device)
    code = _ext.require().read_and_clear_error(torch.device(device).index or 0)
    sys.stderr.write(f"[fused] {what} ok (error word {code})\n")
    sys.stderr.flush()
    if code:
        raise RuntimeError(f"fused {what} reported error code {code}")
_FLAG_BYTES = 256  # sig_ag[8] | sig_rs[8] | arrive[8] | ready[8] | done | pad


class SymmetricWorkspace:
    """This rank's IPC-shared region and its mappings of every peer's region."""

    def __init__(self, group, rows_per_rank: int, width: int, device):
        k = _ext.require()
        self.group = group
        self.tp = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.tp > 8:
            raise ValueError("fused TP collectives support up to 8 ranks")
        self.rows_per_rank = rows_per_rank
        self.width = width
        self.device = torch.device(device)
        self.slot_bytes = rows_per_rank * width * 2
        self.x_off = _FLAG_BYTES
        self.recv_off = self.x_off + 2 * self.slot_bytes
        self.total = self.recv_off + 2 * self.tp * self.slot_bytes
        with torch.cuda.device(self.device):
            self.base, handle = k.symm_alloc(self.total)
            torch.cuda.synchronize()
        handles = [None] * self.tp
        dist.all_gather_object(handles, handle, group=group)
        self.peers = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                self.peers.append(self.base if r == self.rank else k.symm_open(h))
        dist.barrier(group=group)
        self.ag_epoch = 0
        self.rs_epoch = 0
        self.ready_base = 0
        self.done_base = 0
        self.arrive_base = 0
        self.closed = False

    # flag words (u32) inside a region
    def _sig_ag(self, base):
        return base

    def _sig_rs(self, base):
        return base + 32

    def _arrive(self, base):
        return base + 64

    def _ready(self, base):
        return base + 96

    def _done(self, base):
        return base + 128

    def x_slot(self, base, epoch):
        return base + self.x_off + (epoch % 2) * self.slot_bytes

    def recv_slot(self, base, epoch):
        return base + self.recv_off + (epoch % 2) * self.tp * self.slot_bytes

    def fits(self, rows: int, width: int) -> bool:
        return rows == self.rows_per_rank * self.tp and width == self.width

    # --- the two collectives --------------------------------------------------------

    def all_gather_gemm(self, x_local, w, w_mn: bool, n: int):
        """``(all_gather(x_local) @ op(w), gathered x)``; ``op(w)`` is ``w.T`` or ``w`` (``w_mn``)."""
        k = _ext.require()
        self.ag_epoch += 1
        e = self.ag_epoch
        x_local = x_local.contiguous()
        grid = min(148, max(1, x_local.numel() * 2 // (1 << 20)))
        k.ag_publish(x_local, self.x_slot(self.base, e), self.rank, self.tp, e, self._sig_ag(self.base),
                     [self._sig_ag(p) for p in self.peers], self._done(self.base), self.done_base, grid)
        self.done_base += grid
        _debug_check(f"ag_publish epoch {e}", x_local.device)
        t = x_local.shape[0] * self.tp
        xg = torch.empty((t, x_local.shape[1]), dtype=x_local.dtype, device=x_local.device)
        y = torch.empty((t, n), dtype=x_local.dtype, device=x_local.device)
        ggrid = k.fused_grid(t, n, self.tp)
        k.ag_gemm(x_local, xg, [self.x_slot(p, e) for p in self.peers], w, w_mn, y, self.rank, self.tp, e,
                  self._sig_ag(self.base), self._ready(self.base), self.ready_base, ggrid)
        self.ready_base += 2 * ggrid
        _debug_check(f"ag_gemm epoch {e}", x_local.device)
        return y, xg

    def gemm_reduce_scatter(self, h, w, w_mn: bool, n: int):
        """``reduce_scatter_tokens(h @ op(w))`` -> this rank's ``[T/tp, n]`` rows."""
        k = _ext.require()
        self.rs_epoch += 1
        e = self.rs_epoch
        h = h.contiguous()
        t = h.shape[0]
        y = torch.empty((t // self.tp, n), dtype=h.dtype, device=h.device)
        grid = k.fused_grid(t, n, self.tp)
        k.gemm_rs(h, w, w_mn, y, self.rank, self.tp, e, [self.recv_slot(p, e) for p in self.peers],
                  [self._arrive(p) for p in self.peers], [self._sig_rs(p) for p in self.peers],
                  self._arrive(self.base), self._sig_rs(self.base), self.arrive_base,
                  self.recv_slot(self.base, e), grid)
        tiles_per_chunk = (self.rows_per_rank // 128) * ((n + 255) // 256)
        self.arrive_base += 4 * tiles_per_chunk
        _debug_check(f"gemm_rs epoch {e}", h.device)
        return y

    def close(self, *, barrier: bool = True):
        """Unmap the peers' regions and free this one.

        Every rank of the group must have finished its fused kernels first -- a peer may
        still be reading this rank's slots -- so by default the group synchronises before
        anything is unmapped. At a fail-stop safe point (``barrier=False``) no kernel is
        in flight anywhere and the dead peer cannot take part in a barrier.
        """
        if self.closed:
            return
        k = _ext.require()
        torch.cuda.synchronize(self.device)
        if barrier:
            dist.barrier(group=self.group)
        for r, p in enumerate(self.peers):
            if r != self.rank:
                k.symm_close(p)
        k.symm_free(self.base)
        self.closed = True


class _AGLinear(Function):
    @staticmethod
    def forward(ctx, x_local, w, main_grad, ws):
        y, xg = ws.all_gather_gemm(x_local, w, False, w.shape[0])
        ctx.save_for_backward(xg, w)
        ctx.main_grad = main_grad
        ctx.ws = ws
        return y

    @staticmethod
    def backward(ctx, dy):
        xg, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = ctx.ws.gemm_reduce_scatter(dy, w, True, w.shape[1])
        if ctx.main_grad is not None:
            linear_wgrad(dy, xg, out=ctx.main_grad, accumulate=True)
        return dx, None, None, None


class _LinearRS(Function):
    @staticmethod
    def forward(ctx, h, w, main_grad, ws):
        y = ws.gemm_reduce_scatter(h, w, False, w.shape[0])
        ctx.save_for_backward(h, w)
        ctx.main_grad = main_grad
        ctx.ws = ws
        return y

    @staticmethod
    def backward(ctx, dy_local):
        h, w = ctx.saved_tensors
        dh, dyg = ctx.ws.all_gather_gemm(dy_local.contiguous(), w, True, w.shape[1])
        if ctx.main_grad is not None:
            linear_wgrad(dyg, h, out=ctx.main_grad, accumulate=True)
        return dh, None, None, None


def ag_linear(x_local, w, main_grad, ws):
    """Column-parallel SP linear: all-gather over tokens fused into the GEMM."""
    return _AGLinear.apply(x_local, w, main_grad, ws)


def linear_rs(h, w, main_grad, ws):
    """Row-parallel SP linear: reduce-scatter over tokens fused into the GEMM."""
    return _LinearRS.apply(h, w, main_grad, ws)
