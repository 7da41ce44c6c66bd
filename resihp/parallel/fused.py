"""Fused TP linears over NVLink peer memory (csrc/fused_gemm.cu).

With sequence parallelism (tokens sharded between the TP ranks):

* :func:`ag_linear`  -- column-parallel: ``y = all_gather_tokens(x_r) @ w.T`` as one
  AG->GEMM kernel; backward: the input gradient is one GEMM->RS kernel and the weight
  gradient reuses the gathered input the forward kernel assembled.
* :func:`linear_rs`  -- row-parallel: ``y_r = reduce_scatter_tokens(h @ w.T)`` as one
  GEMM->RS kernel; backward: the input gradient is one AG->GEMM kernel over the output
  gradient, whose gathered copy feeds the weight gradient.

Without it (every rank holds every token, the reference's own layout):

* :func:`col_linear_ar` -- column-parallel: a local GEMM forward; backward: the input
  gradient's all-reduce fused into its GEMM (GEMM->AR).
* :func:`row_linear_ar` -- row-parallel: ``y = all_reduce(x @ w.T)`` as one GEMM->AR
  kernel; backward: local GEMMs.

These replace the NCCL collectives of :mod:`resihp.parallel.collectives` (the
baseline; the reference's counterparts are the Megatron ``f`` / ``g`` all-reduce
regions, ``resihp/parallel/tp.py:63-89``). They exchange data through a
:class:`SymmetricWorkspace` per TP group: one CUDA-IPC-shared region per rank holding
the counter words, two AG landing zones, two RS receive buffers and two AR output
landing zones (alternating by call parity). Peers write into each other's regions
(posted P2P stores and release reductions on counters); nothing is multicast.

All ranks of a TP group issue their fused calls in the same order (they follow the same
model code), which is what the epoch counters rely on.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist
from torch.autograd import Function

from ..ops import _ext
from ..ops.gemm import linear, linear_dgrad, linear_wgrad

ENABLED = os.environ.get("RESIHP_FUSED_TP", "1") != "0"
# Largest TP degree that takes the fused kernels; above it NCCL + this package's GEMM.
MAX_DEGREE = int(os.environ.get("RESIHP_FUSED_TP_MAX_DEGREE", "8"))
DEBUG = os.environ.get("RESIHP_FUSED_DEBUG", "0") == "1"

MODE_AG, MODE_RS, MODE_AR = 1, 2, 3
MAX_TP, MAX_RB, MAX_TILES = 8, 256, 8192     # launch.h: kFusedMaxTp, kFusedMaxRb, kFusedMaxTiles
_AG_CNT = 0                                   # byte offsets of the counter words in the flag area
_RS_CNT = _AG_CNT + 4 * MAX_TP * MAX_RB       # two banks by call parity
_AR_CNT = _RS_CNT + 2 * 4 * MAX_TILES
_SEND_CNT = _AR_CNT + 4 * MAX_TILES           # local: finished partial rows per tile (RS, AR)
_OWN_CNT = _SEND_CNT + 4 * MAX_TILES          # local: finished reduced rows per own tile (AR)
_CTRS = _OWN_CNT + 4 * MAX_TILES              # local claim counters: AG tile, AG copy, RS tile, RS copy
_FLAG_BYTES = 176 * 1024
_GUARD_BYTES = 256                            # debug layout: guard bytes after every buffer
_GUARD_VALUE = 0xA5
_U32 = 0xFFFFFFFF


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


class SymmetricWorkspace:
    """This rank's IPC-shared region and its mappings of every peer's region.

    Layout (bytes): counter words (176 KB) | two AG landing zones ``[T, width]`` | two RS
    receive buffers (``[tp][T/128 tiles of this rank's chunk][128 x 256]``, tile-contiguous)
    | two AR output landing zones (``[T/128 x tiles_n][128 x 256]``, tile-contiguous) |
    the RS send buffer (same tiles, local: partial tiles before the copy warps push them
    whole; the AR stages its reduced own tiles there).
    Every fused call's gathered input, reduced output and all-reduced output has the
    model width, so one region serves all projections of a layer and their backward.
    """

    def __init__(self, group, rows_per_rank: int, width: int, device):
        k = _ext.require()
        self.group = group
        self.tp = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.tp > MAX_TP:
            raise ValueError(f"fused TP collectives support up to {MAX_TP} ranks")
        t = rows_per_rank * self.tp
        if rows_per_rank % 128 or rows_per_rank // 128 > MAX_RB:
            raise ValueError("fused TP workspace: rows per rank must be a multiple of 128 (at most 32768)")
        if (t // 128) * ((width + 255) // 256) > MAX_TILES:
            raise ValueError("fused TP workspace: too many output tiles")
        self.rows_per_rank = rows_per_rank
        self.width = width
        self.t = t
        self.device = torch.device(device)
        with torch.cuda.device(self.device):
            self.slices = k.fused_slices(rows_per_rank)
        # every buffer holds [T, width] rows, or (RS send / receive) the same data as whole
        # 128 x 256 tiles, so its size rounds the width up to 256 columns
        self.buf_bytes = t * (-(-width // 256) * 256) * 2
        g = _GUARD_BYTES if DEBUG else 0
        self.stride = self.buf_bytes + g
        self.land_off = _FLAG_BYTES + g
        self.recv_off = self.land_off + 2 * self.stride
        self.out_off = self.recv_off + 2 * self.stride
        self.send_off = self.out_off + 2 * self.stride
        self.total = self.send_off + self.stride
        self.guards = ([_FLAG_BYTES] + [self.land_off + i * self.stride + self.buf_bytes for i in range(7)]) if g else []
        with torch.cuda.device(self.device):
            # a tensor owns the region (freed when the last view of it dies: a caller may
            # still hold the landing-zone view an AG returned)
            self.region, handle = k.symm_region(self.total, self.device.index or 0)
            self.base = self.region.data_ptr()
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
        self.rs_epoch = 0   # RS and AR calls (they share the receive buffers and counters)
        self.ar_epoch = 0
        self.bases = [0, 0, 0, 0]  # claims so far on the AG tile, AG copy, RS tile, RS copy counters
        self.closed = False

    def _buf(self, base, off, epoch):
        return base + off + (epoch % 2) * self.stride

    def _peers(self, tile_ctr: int, copy_ctr: int) -> list[int]:
        """The flat peer description of the next call (see ``decode_peers`` in torch_api.cpp)."""
        head = [self.rank, self.tp, self.rows_per_rank, self.slices, self.ag_epoch if tile_ctr == 0 else self.rs_epoch,
                self.ar_epoch, self.base + _CTRS + 4 * tile_ctr, self.bases[tile_ctr] & _U32,
                self.base + _CTRS + 4 * copy_ctr, self.bases[copy_ctr] & _U32]
        ps = self.peers
        return (head + [self._buf(p, self.land_off, self.ag_epoch) for p in ps] + [p + _AG_CNT for p in ps]
                + [self._buf(p, self.recv_off, self.rs_epoch) for p in ps] + [p + _RS_CNT for p in ps]
                + [self._buf(p, self.out_off, self.ar_epoch) for p in ps] + [p + _AR_CNT for p in ps]
                + [self.base + self.send_off, self.base + _SEND_CNT, self.base + _OWN_CNT])

    def check_guards(self, what: str) -> None:
        """Debug layout: raise if a kernel wrote past any buffer of this region."""
        k = _ext.require()
        for off in self.guards:
            data = k.debug_read_bytes(self.base + off, _GUARD_BYTES)
            if data != bytes([_GUARD_VALUE]) * _GUARD_BYTES:
                raise RuntimeError(f"fused {what}: workspace guard at byte {off} was overwritten")

    def fits(self, rows: int, width: int) -> bool:
        return rows == self.t and width == self.width

    def _after(self, what: str, device, tile_ctr: int, copy_ctr: int, mode: int, n: int, grid: int,
               xg_chunks: int = 0) -> None:
        k = _ext.require()
        self.bases[tile_ctr] += k.fused_tile_claims(self.t, n, grid)
        self.bases[copy_ctr] += k.fused_copy_claims(mode, self.t, n, self.tp, self.slices, xg_chunks, grid)
        _debug_check(what, device)
        if DEBUG:
            self.check_guards(what)

    # --- the three collectives ------------------------------------------------------

    def landing(self, epoch: int, width: int) -> torch.Tensor:
        """This rank's AG landing zone of ``epoch``'s parity as a ``[T, width]`` view."""
        start = self.land_off + (epoch % 2) * self.stride
        return self.region[start:start + self.t * width * 2].view(torch.bfloat16).view(self.t, width)

    def all_gather_gemm(self, x_local, w, w_mn: bool, n: int, *, keep_gathered=True):
        """``(all_gather(x_local) @ op(w), gathered x or None)``; ``op(w)`` is ``w.T`` or ``w`` (``w_mn``).

        ``keep_gathered``: ``True`` copies the gathered input into a new tensor (kept as
        long as the caller wants); ``"landing"`` returns this rank's landing zone itself
        (the kernel adds only the own chunk; valid until the AG call after next, so for
        use right away); ``False`` returns none."""
        k = _ext.require()
        self.ag_epoch += 1
        x_local = x_local.contiguous()
        if keep_gathered == "landing":
            xg, chunks = self.landing(self.ag_epoch, x_local.shape[1]), 1
        elif keep_gathered:
            xg, chunks = torch.empty((self.t, x_local.shape[1]), dtype=x_local.dtype, device=x_local.device), self.tp
        else:
            xg, chunks = None, 0
        y = torch.empty((self.t, n), dtype=x_local.dtype, device=x_local.device)
        grid = k.fused_grid(self.t, n, self.tp)
        k.ag_gemm(x_local, xg, w, w_mn, y, self._peers(0, 1), grid)
        self._after(f"ag_gemm epoch {self.ag_epoch}", x_local.device, 0, 1, MODE_AG, n, grid, chunks)
        return y, xg

    def gemm_reduce_scatter(self, h, w, w_mn: bool, n: int):
        """``reduce_scatter_tokens(h @ op(w))`` -> this rank's ``[T/tp, n]`` rows."""
        k = _ext.require()
        self.rs_epoch += 1
        h = h.contiguous()
        y = torch.empty((self.rows_per_rank, n), dtype=h.dtype, device=h.device)
        grid = k.fused_grid(self.t, n, self.tp)
        k.gemm_rs(h, w, w_mn, y, False, self._peers(2, 3), grid)
        self._after(f"gemm_rs epoch {self.rs_epoch}", h.device, 2, 3, MODE_RS, n, grid)
        return y

    def gemm_all_reduce(self, h, w, w_mn: bool, n: int):
        """``all_reduce(h @ op(w))`` -> the full ``[T, n]`` on every rank."""
        k = _ext.require()
        self.rs_epoch += 1
        self.ar_epoch += 1
        h = h.contiguous()
        y = torch.empty((self.t, n), dtype=h.dtype, device=h.device)
        grid = k.fused_grid(self.t, n, self.tp)
        k.gemm_rs(h, w, w_mn, y, True, self._peers(2, 3), grid)
        self._after(f"gemm_ar epoch {self.ar_epoch}", h.device, 2, 3, MODE_AR, n, grid)
        return y

    def close(self, *, barrier: bool = True):
        """Unmap the peers' regions and free this one.

        Every rank of the group must have finished its fused kernels first -- a peer may
        still be writing into this rank's buffers -- so by default the group
        synchronises before anything is unmapped. At a fail-stop safe point
        (``barrier=False``) no kernel is in flight anywhere and the dead peer cannot
        take part in a barrier.
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
        self.region = None  # freed with its last view
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
        # the gathered output gradient feeds the weight gradient right away: read it in place
        dh, dyg = ctx.ws.all_gather_gemm(dy_local.contiguous(), w, True, w.shape[1],
                                         keep_gathered="landing" if ctx.main_grad is not None else False)
        if ctx.main_grad is not None:
            linear_wgrad(dyg, h, out=ctx.main_grad, accumulate=True)
        return dh, None, None, None


class _ColLinearAR(Function):
    @staticmethod
    def forward(ctx, h, w, main_grad, ws):
        ctx.save_for_backward(h, w)
        ctx.main_grad = main_grad
        ctx.ws = ws
        return linear(h, w)

    @staticmethod
    def backward(ctx, dy):
        h, w = ctx.saved_tensors
        dy = dy.contiguous()
        dh = ctx.ws.gemm_all_reduce(dy, w, True, w.shape[1])
        if ctx.main_grad is not None:
            linear_wgrad(dy, h, out=ctx.main_grad, accumulate=True)
        return dh, None, None, None


class _RowLinearAR(Function):
    @staticmethod
    def forward(ctx, x, w, main_grad, ws):
        ctx.save_for_backward(x, w)
        ctx.main_grad = main_grad
        ctx.ws = ws
        return ws.gemm_all_reduce(x, w, False, w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = linear_dgrad(dy, w)
        if ctx.main_grad is not None:
            linear_wgrad(dy, x, out=ctx.main_grad, accumulate=True)
        return dx, None, None, None


def ag_linear(x_local, w, main_grad, ws):
    """Column-parallel SP linear: all-gather over tokens fused into the GEMM."""
    return _AGLinear.apply(x_local, w, main_grad, ws)


def linear_rs(h, w, main_grad, ws):
    """Row-parallel SP linear: reduce-scatter over tokens fused into the GEMM."""
    return _LinearRS.apply(h, w, main_grad, ws)


def col_linear_ar(h, w, main_grad, ws):
    """Column-parallel linear without SP: the input gradient's all-reduce fused into its GEMM."""
    return _ColLinearAR.apply(h, w, main_grad, ws)


def row_linear_ar(x, w, main_grad, ws):
    """Row-parallel linear without SP: the output all-reduce fused into the GEMM."""
    return _RowLinearAR.apply(x, w, main_grad, ws)
