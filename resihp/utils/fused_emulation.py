"""The fused TP kernels on one GPU, with the peers emulated by local buffers.

A fused launch of group rank 0 out of ``tp`` normally pushes into its peers' workspaces
over NVLink and waits on counters the peers raise in its own workspace. Here every
"peer" workspace is a second region on the same device with the same layout, the data
each peer would have pushed into rank 0 is written there beforehand and every counter
rank 0 waits on is preset far ahead -- so the launch runs alone, waits for nothing and
can be checked against torch, timed, or captured by a profiler on a single GPU. (Two
kernels that wait on each other never run as separate launches on one GPU; here
nothing is waited on.) Rank 0's own pushes land in the emulated peers' regions, where a
test can check them.

    from resihp.utils.fused_emulation import Emulation
    em = Emulation(tokens=4096, width=2048, tp=2)
    y = em.all_gather_gemm(w)          # y = gather(x) @ w.T, rank 0's view
"""

from __future__ import annotations

import torch

from ..ops import _ext
from ..parallel import fused

_FAR = 1 << 30  # a counter value no launch of a test reaches


class Emulation:
    """``tp`` workspaces on one device laid out like :class:`~resihp.parallel.fused.
    SymmetricWorkspace`; launches run as group rank 0."""

    def __init__(self, tokens: int, width: int, *, tp: int = 2, seed: int = 0, device="cuda"):
        self.kx = _ext.require()
        self.dev = torch.device(device)
        self.tp, self.t, self.width = tp, tokens, width
        self.rpr = tokens // tp
        g = torch.Generator(device=self.dev).manual_seed(seed)
        self.gen = g
        with torch.cuda.device(self.dev):
            self.slices = self.kx.fused_slices(self.rpr)
        self.buf_bytes = tokens * (-(-width // 256) * 256) * 2  # as SymmetricWorkspace
        self.land_off = fused._FLAG_BYTES
        self.recv_off = self.land_off + 2 * self.buf_bytes
        self.out_off = self.recv_off + 2 * self.buf_bytes
        self.send_off = self.out_off + 2 * self.buf_bytes
        total = self.send_off + self.buf_bytes
        self.regions = [torch.zeros(total, dtype=torch.uint8, device=self.dev) for _ in range(tp)]
        self.bases = [r.data_ptr() for r in self.regions]
        self.epochs = {"ag": 0, "rs": 0, "ar": 0}
        self.claims = [0, 0, 0, 0]
        self.x = torch.randn(tokens, width, device=self.dev, generator=g).bfloat16()  # every rank's chunk, stacked
        # rank 0's waits pass at once; the peers' counters start at zero (rank 0 raises them)
        self.u32(0, fused._AG_CNT, fused.MAX_TP * fused.MAX_RB).view(fused.MAX_TP, fused.MAX_RB)[1:].fill_(_FAR)
        self.u32(0, fused._RS_CNT, 2 * fused.MAX_TILES).fill_(_FAR)
        self.u32(0, fused._AR_CNT, fused.MAX_TILES).fill_(_FAR)
        for parity in range(2):  # the peers' chunks already in rank 0's landing zones
            self.buf(0, self.land_off, parity, (tokens, width))[self.rpr:].copy_(self.x[self.rpr:])

    # --- views into the emulated workspaces ---------------------------------------------
    def u32(self, rank, off, count):
        return self.regions[rank][off:off + 4 * count].view(torch.int32)

    def recv_tiles(self, rank, parity, n):
        """Rank ``rank``'s receive buffer as ``[tp, tiles of a chunk, 128, 256]``."""
        tiles = (self.rpr // 128) * (-(-n // 256))
        return self.buf(rank, self.recv_off, parity, (self.tp * tiles * 128, 256)).view(self.tp, tiles, 128, 256)

    def out_tiles(self, rank, parity, n):
        """Rank ``rank``'s AR output landing zone as ``[T/128 x tiles_n, 128, 256]`` tiles."""
        tiles = (self.t // 128) * (-(-n // 256))
        return self.buf(rank, self.out_off, parity, (tiles * 128, 256)).view(tiles, 128, 256)

    def to_tiles(self, rows_x_n):
        """``[rows, n]`` rows as the kernels' tile-contiguous ``[tiles, 128, 256]`` (tile =
        128-row block major, then 256-column block; columns past n zero)."""
        r, n = rows_x_n.shape
        tn = -(-n // 256)
        padded = torch.zeros(r, tn * 256, dtype=rows_x_n.dtype, device=rows_x_n.device)
        padded[:, :n] = rows_x_n
        return padded.view(r // 128, 128, tn, 256).permute(0, 2, 1, 3).reshape(-1, 128, 256)

    def from_tiles(self, tiles, n):
        """Inverse of :meth:`to_tiles` (``[tiles, 128, 256]`` -> ``[rpr, n]``)."""
        tn = -(-n // 256)
        t = tiles.view(-1, tn, 128, 256).permute(0, 2, 1, 3).reshape(-1, tn * 256)
        return t[:, :n]

    def buf(self, rank, off, parity, shape):
        start = off + parity * self.buf_bytes
        n = shape[0] * shape[1]
        return self.regions[rank][start:start + 2 * n].view(torch.bfloat16).view(shape)

    def _peers(self, tile_ctr, copy_ctr, epoch):
        head = [0, self.tp, self.rpr, self.slices, epoch, self.epochs["ar"], self.bases[0] + fused._CTRS + 4 * tile_ctr,
                self.claims[tile_ctr] & fused._U32, self.bases[0] + fused._CTRS + 4 * copy_ctr,
                self.claims[copy_ctr] & fused._U32]
        bs = self.bases
        return (head + [b + self.land_off + (self.epochs["ag"] % 2) * self.buf_bytes for b in bs]
                + [b + fused._AG_CNT for b in bs]
                + [b + self.recv_off + (self.epochs["rs"] % 2) * self.buf_bytes for b in bs]
                + [b + fused._RS_CNT for b in bs]
                + [b + self.out_off + (self.epochs["ar"] % 2) * self.buf_bytes for b in bs]
                + [b + fused._AR_CNT for b in bs]
                + [bs[0] + self.send_off, bs[0] + fused._SEND_CNT, bs[0] + fused._OWN_CNT])

    def _advance(self, tile_ctr, copy_ctr, mode, n, grid, xg_chunks):
        self.claims[tile_ctr] += self.kx.fused_tile_claims(self.t, n, grid)
        self.claims[copy_ctr] += self.kx.fused_copy_claims(mode, self.t, n, self.tp, self.slices, xg_chunks, grid)

    # --- the three launches (rank 0) ------------------------------------------------------
    def all_gather_gemm(self, w, *, w_mn=False, keep_gathered=True):
        """``(y, xg)`` of rank 0's AG->GEMM: ``y = gather(x) @ op(w)`` (``keep_gathered`` as
        in :meth:`~resihp.parallel.fused.SymmetricWorkspace.all_gather_gemm`)."""
        self.epochs["ag"] += 1
        n = w.shape[1] if w_mn else w.shape[0]
        if keep_gathered == "landing":
            xg, chunks = self.buf(0, self.land_off, self.epochs["ag"] % 2, (self.t, self.width)), 1
        elif keep_gathered:
            xg, chunks = torch.empty(self.t, self.width, device=self.dev, dtype=torch.bfloat16), self.tp
        else:
            xg, chunks = None, 0
        y = torch.empty(self.t, n, device=self.dev, dtype=torch.bfloat16)
        grid = self.kx.fused_grid(self.t, n, self.tp)
        self.kx.ag_gemm(self.x[:self.rpr], xg, w, w_mn, y, self._peers(0, 1, self.epochs["ag"]), grid)
        self._advance(0, 1, fused.MODE_AG, n, grid, chunks)
        return y, xg

    def preset_partials(self, h_peers, w_peers, *, w_mn=False, all_reduce=False):
        """Write what every peer would push into rank 0 for an RS (or AR) launch: each
        peer's bf16 partial of rank 0's rows, in both parities (and, for an AR, every
        other owner's reduced rows in rank 0's output landing zone). Returns the FP32
        reference of the launch's output."""
        n = w_peers[0].shape[1] if w_mn else w_peers[0].shape[0]
        op = (lambda w: w.float()) if w_mn else (lambda w: w.float().t())
        parts = [h.float() @ op(w) for h, w in zip(h_peers, w_peers)]
        for parity in range(2):
            recv = self.recv_tiles(0, parity, n)
            for src in range(1, self.tp):
                recv[src].copy_(self.to_tiles(parts[src][:self.rpr].bfloat16()))
        if not all_reduce:
            own = parts[0][:self.rpr]
            return own + sum(parts[src][:self.rpr].bfloat16().float() for src in range(1, self.tp))
        full = parts[0].clone()
        for src in range(1, self.tp):
            full += parts[src].bfloat16().float()
        per_chunk = (self.rpr // 128) * (-(-n // 256))
        for parity in range(2):  # every other owner's reduced tiles, tile-contiguous
            self.out_tiles(0, parity, n)[per_chunk:].copy_(self.to_tiles(full.bfloat16())[per_chunk:])
        return full

    def gemm_reduce_scatter(self, h, w, *, w_mn=False):
        self.epochs["rs"] += 1
        n = w.shape[1] if w_mn else w.shape[0]
        y = torch.empty(self.rpr, n, device=self.dev, dtype=torch.bfloat16)
        grid = self.kx.fused_grid(self.t, n, self.tp)
        self.kx.gemm_rs(h, w, w_mn, y, False, self._peers(2, 3, self.epochs["rs"]), grid)
        self._advance(2, 3, fused.MODE_RS, n, grid, 0)
        return y

    def gemm_all_reduce(self, h, w, *, w_mn=False):
        self.epochs["rs"] += 1
        self.epochs["ar"] += 1
        n = w.shape[1] if w_mn else w.shape[0]
        y = torch.empty(self.t, n, device=self.dev, dtype=torch.bfloat16)
        grid = self.kx.fused_grid(self.t, n, self.tp)
        self.kx.gemm_rs(h, w, w_mn, y, True, self._peers(2, 3, self.epochs["rs"]), grid)
        self._advance(2, 3, fused.MODE_AR, n, grid, 0)
        return y


class AgSession:
    """Repeated emulated AG->GEMM launches (one set of buffers), for timing and captures."""

    def __init__(self, tokens: int, k: int, n: int, *, tp: int = 2, keep_gathered: bool = True, device="cuda"):
        self.em = Emulation(tokens, k, tp=tp, device=device)
        self.w = (torch.randn(n, k, device=device) / k**0.5).bfloat16()
        self.keep = keep_gathered

    def launch(self):
        return self.em.all_gather_gemm(self.w, keep_gathered=self.keep)[0]


class RsSession:
    """Repeated emulated GEMM->RS (or GEMM->AR) launches of rank 0, for timing and captures."""

    def __init__(self, tokens: int, k: int, n: int, *, tp: int = 2, all_reduce: bool = False, device="cuda"):
        self.em = Emulation(tokens, n, tp=tp, device=device)
        self.h = torch.randn(tokens, k, device=device).bfloat16()
        self.w = (torch.randn(n, k, device=device) / k**0.5).bfloat16()
        self.all_reduce = all_reduce

    def launch(self):
        if self.all_reduce:
            return self.em.gemm_all_reduce(self.h, self.w)
        return self.em.gemm_reduce_scatter(self.h, self.w)
