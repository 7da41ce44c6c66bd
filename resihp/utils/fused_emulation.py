"""The fused TP kernels on one GPU, with the peers emulated by local buffers.

A fused AG->GEMM or GEMM->RS launch of group rank 0 out of ``tp`` normally reads its
peers' symmetric buffers over NVLink and waits for their flag words. Here every peer
buffer is a second buffer on the same device, filled with what that peer would have
published, and every flag word the kernel waits on is set before the launch -- so the
launch runs alone, waits for nothing, and can be checked against torch or captured by
a profiler on a single GPU. (Two kernels that wait on each other never run as separate
launches on one GPU; here nothing is waited on.)

    from resihp.utils.fused_emulation import emulate_ag, emulate_rs
    y, want = emulate_ag(tokens=4096, k=2048, n=3072, tp=2)
"""

from __future__ import annotations

import torch

from ..ops import _ext


def _u32(count, device, fill=0):
    return torch.full((count,), fill, dtype=torch.int32, device=device)


def emulate_ag(tokens: int, k: int, n: int, *, tp: int = 2, epoch: int = 1, seed: int = 0, device="cuda",
               variant: int = 0):
    """``(y, reference)`` of one emulated AG->GEMM launch of rank 0: ``y = gather(x) @ w.T``."""
    kx = _ext.require()
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    rows = tokens // tp
    chunks = [torch.randn(rows, k, device=dev, generator=g).bfloat16() for _ in range(tp)]
    w = (torch.randn(n, k, device=dev, generator=g) / k**0.5).bfloat16()
    slots = [torch.empty_like(chunks[0])] + [c.clone() for c in chunks[1:]]  # peers already published
    xg = torch.empty(tokens, k, device=dev, dtype=torch.bfloat16)
    y = torch.empty(tokens, n, device=dev, dtype=torch.bfloat16)
    sig = _u32(8, dev)
    sig[1:tp] = epoch                      # every peer announced this epoch
    peer_sig = [_u32(8, dev) for _ in range(tp)]  # where this rank's announcement lands
    pub = _u32(1, dev)
    ready = _u32(tp, dev)
    rb_ready = _u32(tokens // 128, dev)
    grid = kx.fused_grid(tokens, n, tp)
    kx.ag_gemm(chunks[0], slots[0].data_ptr(), [s.data_ptr() for s in slots], xg, w, False, y, 0, tp, epoch,
               sig.data_ptr(), [p.data_ptr() for p in peer_sig], pub.data_ptr(), 0, ready.data_ptr(), 0, grid,
               variant, rb_ready.data_ptr(), 0)
    ref = torch.cat(chunks).float() @ w.float().t()
    return y, ref, xg, torch.cat(chunks)


def emulate_rs(tokens: int, k: int, n: int, *, tp: int = 2, epoch: int = 1, seed: int = 0, device="cuda",
               variant: int = 0):
    """``(y_r, reference)`` of one emulated GEMM->RS launch of rank 0: rows ``[0, T/tp)`` of
    ``sum over ranks of h_rank @ w_rank.T``, the peers' partials preset in local buffers."""
    kx = _ext.require()
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    rows = tokens // tp
    hs = [torch.randn(tokens, k, device=dev, generator=g).bfloat16() for _ in range(tp)]
    ws = [(torch.randn(n, k, device=dev, generator=g) / k**0.5).bfloat16() for _ in range(tp)]
    partials = [(h.float() @ w.float().t()).bfloat16() for h, w in zip(hs, ws)]  # what each peer publishes
    parts = [torch.empty(tokens, n, device=dev, dtype=torch.bfloat16)] + partials[1:]
    tiles = (tokens // 128) * ((n + 255) // 256)
    own_flags = _u32(tiles, dev)
    peer_flags = [own_flags] + [_u32(tiles, dev, 4 * epoch) for _ in range(1, tp)]  # every peer tile is final
    recv = torch.empty(tp, rows, n, device=dev, dtype=torch.bfloat16)
    y = torch.empty(rows, n, device=dev, dtype=torch.bfloat16)
    grid = kx.fused_grid(tokens, n, tp)
    kx.gemm_rs(hs[0], ws[0], False, y, 0, tp, epoch, parts[0].data_ptr(), [p.data_ptr() for p in parts],
               own_flags.data_ptr(), [f.data_ptr() for f in peer_flags], recv.data_ptr(), grid, variant)
    own = hs[0][:rows].float() @ ws[0].float().t()
    ref = own + sum(p[:rows].float() for p in partials[1:])
    return y, ref


class AgSession:
    """Repeated emulated AG->GEMM launches of rank 0 on one set of buffers, with the
    epoch and the counter bases advanced per launch as the real workspace advances them
    (so every launch waits for its own pulls); the peers' announcements are preset far
    ahead. For timing and profiler captures."""

    def __init__(self, tokens: int, k: int, n: int, *, tp: int = 2, variant: int = 0, device="cuda"):
        self.kx = _ext.require()
        dev = torch.device(device)
        rows = tokens // tp
        self.tp, self.n, self.t, self.variant = tp, n, tokens, variant
        self.chunks = [torch.randn(rows, k, device=dev).bfloat16() for _ in range(tp)]
        self.w = (torch.randn(n, k, device=dev) / k**0.5).bfloat16()
        self.slots = [torch.empty_like(self.chunks[0])] + [c.clone() for c in self.chunks[1:]]
        self.xg = torch.empty(tokens, k, device=dev, dtype=torch.bfloat16)
        self.y = torch.empty(tokens, n, device=dev, dtype=torch.bfloat16)
        self.sig = _u32(8, dev)
        self.sig[1:tp] = 1 << 30
        self.peer_sig = [_u32(8, dev) for _ in range(tp)]
        self.pub, self.ready, self.rb_ready = _u32(1, dev), _u32(tp, dev), _u32(tokens // 128, dev)
        self.grid = self.kx.fused_grid(tokens, n, tp)
        self.epoch = self.pub_base = self.ready_base = self.rb_base = 0

    def launch(self):
        kx = self.kx
        self.epoch += 1
        kx.ag_gemm(self.chunks[0], self.slots[0].data_ptr(), [s.data_ptr() for s in self.slots], self.xg, self.w,
                   False, self.y, 0, self.tp, self.epoch, self.sig.data_ptr(), [p.data_ptr() for p in self.peer_sig],
                   self.pub.data_ptr(), self.pub_base, self.ready.data_ptr(), self.ready_base, self.grid,
                   self.variant, self.rb_ready.data_ptr(), self.rb_base)
        step = kx.fused_counter_step(self.grid, self.variant)
        self.pub_base += step
        if self.variant == 0:
            self.ready_base += step
        else:
            self.rb_base += kx.fused_block_step(self.t, self.n, self.tp, self.grid)
        return self.y


class RsSession:
    """Repeated emulated GEMM->RS launches of rank 0 (peer tile flags preset far ahead)."""

    def __init__(self, tokens: int, k: int, n: int, *, tp: int = 2, variant: int = 0, device="cuda"):
        self.kx = _ext.require()
        dev = torch.device(device)
        rows = tokens // tp
        self.tp, self.variant = tp, variant
        self.h = torch.randn(tokens, k, device=dev).bfloat16()
        self.w = (torch.randn(n, k, device=dev) / k**0.5).bfloat16()
        self.parts = [torch.empty(tokens, n, device=dev, dtype=torch.bfloat16) for _ in range(tp)]
        tiles = (tokens // 128) * ((n + 255) // 256)
        self.own_flags = _u32(tiles, dev)
        self.peer_flags = [self.own_flags] + [_u32(tiles, dev, 1 << 30) for _ in range(1, tp)]
        self.recv = torch.empty(tp, rows, n, device=dev, dtype=torch.bfloat16)
        self.y = torch.empty(rows, n, device=dev, dtype=torch.bfloat16)
        self.grid = self.kx.fused_grid(tokens, n, tp)
        self.epoch = 0

    def launch(self):
        self.epoch += 1
        self.kx.gemm_rs(self.h, self.w, False, self.y, 0, self.tp, self.epoch, self.parts[0].data_ptr(),
                        [p.data_ptr() for p in self.parts], self.own_flags.data_ptr(),
                        [f.data_ptr() for f in self.peer_flags], self.recv.data_ptr(), self.grid, self.variant)
        return self.y
