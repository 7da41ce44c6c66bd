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
