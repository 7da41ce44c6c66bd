"""Fused AG->GEMM / GEMM->RS / GEMM->AR kernels on ONE GPU, peers emulated by local buffers.

Group rank 0 launches; the "peers" are second workspaces on the same device whose data
and counters are preset as if the peers had already pushed (see
``resihp.utils.fused_emulation``), so no launch waits on another. Checked for TP degrees
2, 4 and 8 against an FP32 torch product: the output, the gathered input kept for the
backward pass, and what rank 0 itself pushed into the peers' workspaces -- its chunk in
every peer's landing zone (AG), its partial tiles in each owner's receive buffer (RS),
its reduced tiles in every peer's output landing zone (AR) -- with the counter
increments the peers would wait on.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

T, K, N = 1024, 512, 768


def _rel(a, b):
    return ((a.float() - b).norm() / b.norm()).item()


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_emulated_ag_gemm(tp):
    from resihp.ops import check_device_errors
    from resihp.parallel import fused
    from resihp.utils.fused_emulation import Emulation

    em = Emulation(T, K, tp=tp, seed=tp)
    w = (torch.randn(N, K, device="cuda") / K**0.5).bfloat16()
    for call in (1, 2, 3):
        y, xg = em.all_gather_gemm(w)
        torch.cuda.synchronize()
        check_device_errors(0)
        assert torch.equal(xg, em.x)  # the whole gathered input, for the weight gradient
        assert _rel(y, em.x.float() @ w.float().t()) < 1e-2
        parity = call % 2
        blocks = em.rpr // 128
        for peer in range(1, tp):
            land = em.buf(peer, em.land_off, parity, (T, K))
            assert torch.equal(land[:em.rpr], em.x[:em.rpr])  # rank 0's chunk, rows 0..T/tp
            cnt = em.u32(peer, fused._AG_CNT, fused.MAX_TP * fused.MAX_RB).view(fused.MAX_TP, fused.MAX_RB)
            assert torch.equal(cnt[0, :blocks].cpu(), torch.full((blocks,), em.slices * call, dtype=torch.int32))
            assert int(cnt[0, blocks:].abs().sum()) == 0


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_emulated_ag_gemm_mn_weight(tp):
    """The backward form (``w`` read N-major: ``dy_gathered @ w``), without a gathered copy
    and with the landing zone itself as the gathered input (only the own chunk added)."""
    from resihp.ops import check_device_errors
    from resihp.utils.fused_emulation import Emulation

    em = Emulation(T, K, tp=tp, seed=3 * tp)
    w = (torch.randn(K, N, device="cuda") / K**0.5).bfloat16()
    y, xg = em.all_gather_gemm(w, w_mn=True, keep_gathered=False)
    torch.cuda.synchronize()
    check_device_errors(0)
    assert xg is None and _rel(y, em.x.float() @ w.float()) < 1e-2
    y, land = em.all_gather_gemm(w, w_mn=True, keep_gathered="landing")
    torch.cuda.synchronize()
    check_device_errors(0)
    assert torch.equal(land, em.x) and _rel(y, em.x.float() @ w.float()) < 1e-2


@pytest.mark.parametrize("all_reduce", [False, True], ids=["rs", "ar"])
@pytest.mark.parametrize("tp", [2, 4, 8])
def test_emulated_gemm_rs_ar(tp, all_reduce):
    from resihp.ops import check_device_errors
    from resihp.parallel import fused
    from resihp.utils.fused_emulation import Emulation

    em = Emulation(T, N, tp=tp, seed=10 * tp)
    g = torch.Generator(device="cuda").manual_seed(5 + tp)
    hs = [torch.randn(T, K, device="cuda", generator=g).bfloat16() for _ in range(tp)]
    ws = [(torch.randn(N, K, device="cuda", generator=g) / K**0.5).bfloat16() for _ in range(tp)]
    ref = em.preset_partials(hs, ws, all_reduce=all_reduce)
    tiles_n = (N + 255) // 256
    per_chunk = (em.rpr // 128) * tiles_n
    from resihp.ops import linear

    mine = linear(hs[0], ws[0])  # this package's GEMM: the same accumulation order as the fused kernel
    for call in (1, 2):
        y = em.gemm_all_reduce(hs[0], ws[0]) if all_reduce else em.gemm_reduce_scatter(hs[0], ws[0])
        torch.cuda.synchronize()
        check_device_errors(0)
        assert y.shape[0] == (T if all_reduce else em.rpr)
        assert _rel(y, ref) < 1e-2
        parity = call % 2
        for owner in range(1, tp):
            # rank 0's partial of the owner's rows, in the owner's receive buffer slot 0
            # (tile-contiguous: 128 x 256 tiles)
            recv = em.recv_tiles(owner, parity, N)
            assert torch.equal(em.from_tiles(recv[0], N), mine[owner * em.rpr:(owner + 1) * em.rpr])
            bank = em.u32(owner, fused._RS_CNT, 2 * fused.MAX_TILES).view(2, fused.MAX_TILES)[call % 2]
            assert torch.equal(bank[:per_chunk].cpu(), torch.full((per_chunk,), 1, dtype=torch.int32))
            if all_reduce:
                out = em.from_tiles(em.out_tiles(owner, parity, N), N)  # tile-contiguous landing zone
                assert torch.equal(out[:em.rpr], y[:em.rpr])  # rank 0's reduced rows pushed to every peer
                arc = em.u32(owner, fused._AR_CNT, fused.MAX_TILES)
                grid = em.kx.fused_grid(T, N, tp)
                slices = em.kx.fused_red_slices(T, N, tp, grid)  # each reduced row slice is counted
                assert torch.equal(arc[:per_chunk].cpu(), torch.full((per_chunk,), slices * call, dtype=torch.int32))
