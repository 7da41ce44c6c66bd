"""Fused sequence-parallel TP linears over NVLink peer memory (csrc/fused_gemm.cu).

* :func:`ag_linear`  -- column-parallel: ``y = all_gather_tokens(x_r) @ w.T`` as one
  AG->GEMM kernel; backward: the input gradient is one GEMM->RS kernel and the weight
  gradient reuses the gathered input the forward kernel left in its gather buffer.
* :func:`linear_rs`  -- row-parallel: ``y_r = reduce_scatter_tokens(h @ w.T)`` as one
  GEMM->RS kernel; backward: the input gradient is one AG->GEMM kernel over the output
  gradient, whose gathered copy feeds the weight gradient.

Both replace the NCCL pair ``gather_tokens`` / ``scatter_tokens`` of
:mod:`resihp.parallel.collectives` (the baseline; the reference's counterparts are the
Megatron ``f`` / ``g`` all-reduce regions, ``resihp/parallel/tp.py:63-89``). They exchange data through a
:class:`SymmetricWorkspace` per TP group: one CUDA-IPC-shared region per rank holding
the cross-GPU flag words, two publish slots for the AG input and two partial buffers
for the RS (alternating by call parity), plus a local receive buffer. Peers only ever
read each other's regions (P2P loads) and write each other's flag words; nothing in the
workspace is multicast.

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
# Largest TP degree that takes the fused kernels. Above it the NCCL collectives + this
# package's GEMM are used: in these kernels every CTA pulls a slice of every peer chunk
# with register-staged loads, which keeps too few bytes in flight once the per-rank
# chunk is small and the peers many (measured slower than NCCL at TP8).
MAX_DEGREE = int(os.environ.get("RESIHP_FUSED_TP_MAX_DEGREE", "2"))
# Kernel variant for TP > 2 (six copy warps with sixteen loads in flight each, per-row-block
# readiness in the AG, first-ready peer order in the RS). Off until measured on GPUs.
ROW_BLOCK_VARIANT = os.environ.get("RESIHP_FUSED_TP_V3", "0") == "1"
_RB_READY = 256  # byte offset of the per-row-block ready counters in the flag area
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


_MAX_TILES = 8192             # per-tile flags of the RS partial buffer
_FLAG_BYTES = 4096 + 4 * _MAX_TILES
_GUARD_BYTES = 256            # debug layout: guard bytes after every buffer
_GUARD_VALUE = 0xA5


class SymmetricWorkspace:
    """This rank's IPC-shared region and its mappings of every peer's region.

    Layout (bytes): flag words | two AG publish slots ``[T/tp, width]`` | two RS partial
    buffers ``[T, width]`` | one RS receive buffer ``[tp, T/tp, width]``. The AG input and
    the RS output of every fused call have the model width, so one region serves all four
    projections of a layer and their backward passes.
    """

    def __init__(self, group, rows_per_rank: int, width: int, device):
        k = _ext.require()
        self.group = group
        self.tp = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.tp > 8:
            raise ValueError("fused TP collectives support up to 8 ranks")
        t = rows_per_rank * self.tp
        if (t // 128) * ((width + 255) // 256) > _MAX_TILES:
            raise ValueError("fused TP workspace: too many output tiles")
        if _RB_READY + 4 * (t // 128) > 4096:
            raise ValueError("fused TP workspace: too many row blocks for the flag area")
        self.variant = 1 if (self.tp > 2 and ROW_BLOCK_VARIANT) else 0
        self.rows_per_rank = rows_per_rank
        self.width = width
        self.device = torch.device(device)
        self.slot_bytes = rows_per_rank * width * 2
        self.part_bytes = t * width * 2
        # debug builds of the layout put a guard after every buffer (none otherwise, so
        # the production layout is unchanged)
        g = _GUARD_BYTES if DEBUG else 0
        self.slot_off = _FLAG_BYTES + g
        self.slot_stride = self.slot_bytes + g
        self.part_off = self.slot_off + 2 * self.slot_stride
        self.part_stride = self.part_bytes + g
        self.recv_off = self.part_off + 2 * self.part_stride
        self.total = self.recv_off + self.tp * self.slot_bytes + g
        self.guards = [_FLAG_BYTES] + [self.slot_off + i * self.slot_stride + self.slot_bytes for i in range(2)] + [
            self.part_off + i * self.part_stride + self.part_bytes for i in range(2)] + [self.total - g] if g else []
        with torch.cuda.device(self.device):
            self.base, handle = k.symm_alloc(self.total)
            for off in self.guards:
                k.debug_fill_bytes(self.base + off, _GUARD_BYTES, _GUARD_VALUE)
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
        self.pub_base = 0
        self.ready_base = 0
        self.rb_base = 0
        self.closed = False

    # flag words (u32) inside a region
    def _sig_ag(self, base):
        return base

    def _pub(self, base):
        return base + 64

    def _ready(self, base):
        return base + 128

    def _tile_flags(self, base):
        return base + 4096

    def _slot(self, base, epoch):
        return base + self.slot_off + (epoch % 2) * self.slot_stride

    def _part(self, base, epoch):
        return base + self.part_off + (epoch % 2) * self.part_stride

    def check_guards(self, what: str) -> None:
        """Debug layout: raise if a kernel wrote past any buffer of this region."""
        k = _ext.require()
        for off in self.guards:
            data = k.debug_read_bytes(self.base + off, _GUARD_BYTES)
            if data != bytes([_GUARD_VALUE]) * _GUARD_BYTES:
                raise RuntimeError(f"fused {what}: workspace guard at byte {off} was overwritten")

    def fits(self, rows: int, width: int) -> bool:
        return rows == self.rows_per_rank * self.tp and width == self.width

    # --- the two collectives --------------------------------------------------------

    def all_gather_gemm(self, x_local, w, w_mn: bool, n: int):
        """``(all_gather(x_local) @ op(w), gathered x)``; ``op(w)`` is ``w.T`` or ``w`` (``w_mn``)."""
        k = _ext.require()
        self.ag_epoch += 1
        e = self.ag_epoch
        x_local = x_local.contiguous()
        t = x_local.shape[0] * self.tp
        xg = torch.empty((t, x_local.shape[1]), dtype=x_local.dtype, device=x_local.device)
        y = torch.empty((t, n), dtype=x_local.dtype, device=x_local.device)
        grid = k.fused_grid(t, n, self.tp)
        k.ag_gemm(x_local, self._slot(self.base, e), [self._slot(p, e) for p in self.peers], xg, w, w_mn, y,
                  self.rank, self.tp, e, self._sig_ag(self.base), [self._sig_ag(p) for p in self.peers],
                  self._pub(self.base), self.pub_base, self._ready(self.base), self.ready_base, grid,
                  self.variant, self.base + _RB_READY, self.rb_base)
        step = k.fused_counter_step(grid, self.variant)  # the kernel's own per-launch counter increments
        self.pub_base += step
        if self.variant == 0:
            self.ready_base += step
        else:
            self.rb_base += k.fused_block_step(t, n, self.tp, grid)
        _debug_check(f"ag_gemm epoch {e}", x_local.device)
        if DEBUG:
            self.check_guards(f"ag_gemm epoch {e}")
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
        k.gemm_rs(h, w, w_mn, y, self.rank, self.tp, e, self._part(self.base, e),
                  [self._part(p, e) for p in self.peers], self._tile_flags(self.base),
                  [self._tile_flags(p) for p in self.peers], self.base + self.recv_off, grid, self.variant)
        _debug_check(f"gemm_rs epoch {e}", h.device)
        if DEBUG:
            self.check_guards(f"gemm_rs epoch {e}")
        return y

    def close(self, *, barrier: bool = True):
        """Unmap the peers' regions and free this one.

        Every rank of the group must have finished its fused kernels first -- a peer may
        still be reading this rank's buffers -- so by default the group synchronises
        before anything is unmapped. At a fail-stop safe point (``barrier=False``) no
        kernel is in flight anywhere and the dead peer cannot take part in a barrier.
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
