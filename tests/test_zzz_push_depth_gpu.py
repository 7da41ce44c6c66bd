"""Pipelined RS / AR partial-tile pushes (``RESIHP_PUSH_DEPTH=2``) on ONE GPU, peers emulated.

With push depth 2 a copy thread issues a partial-tile push and counts the previous one
only once it has landed (``bulk_push_issue`` + ``cp.async.bulk.wait_group``), paying
every owed count before it waits on a peer. This checks, in the single-GPU emulation,
that the output equals the default path's bit for bit, that rank 0's partial tiles
reach every owner's receive buffer and that every owner's tile counter is incremented
exactly once per call. Opt-in (``RESIHP_TEST_PUSH_DEPTH=1``) until the path has run on
a GPU; it runs last in the GPU tier.
"""

import os

import pytest
import torch

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(os.environ.get("RESIHP_TEST_PUSH_DEPTH") != "1",
                       reason="opt-in: set RESIHP_TEST_PUSH_DEPTH=1 to run the pipelined push path"),
]

T, K, N = 1024, 512, 768


@pytest.mark.parametrize("all_reduce", [False, True], ids=["rs", "ar"])
@pytest.mark.parametrize("tp", [2, 4])
def test_pipelined_pushes_match_the_default_path(tp, all_reduce):
    from resihp.ops import check_device_errors
    from resihp.parallel import fused
    from resihp.utils.fused_emulation import Emulation

    def run(depth):
        em = Emulation(T, N, tp=tp, seed=10 * tp)
        g = torch.Generator(device="cuda").manual_seed(5 + tp)
        hs = [torch.randn(T, K, device="cuda", generator=g).bfloat16() for _ in range(tp)]
        ws = [(torch.randn(N, K, device="cuda", generator=g) / K**0.5).bfloat16() for _ in range(tp)]
        em.preset_partials(hs, ws, all_reduce=all_reduce)
        em.kx.set_fused_push_depth(depth)
        try:
            outs = []
            for call in (1, 2):
                y = em.gemm_all_reduce(hs[0], ws[0]) if all_reduce else em.gemm_reduce_scatter(hs[0], ws[0])
                torch.cuda.synchronize()
                check_device_errors(0)
                per_chunk = (em.rpr // 128) * ((N + 255) // 256)
                for owner in range(1, tp):
                    bank = em.u32(owner, fused._RS_CNT, 2 * fused.MAX_TILES).view(2, fused.MAX_TILES)[call % 2]
                    assert torch.equal(bank[:per_chunk].cpu(), torch.full((per_chunk,), 1, dtype=torch.int32))
                recv = [em.from_tiles(em.recv_tiles(o, call % 2, N)[0], N) for o in range(1, tp)]
                outs.append((y.clone(), [r.clone() for r in recv]))
            return outs
        finally:
            em.kx.set_fused_push_depth(1)

    base, piped = run(1), run(2)
    for (y1, r1), (y2, r2) in zip(base, piped):
        assert torch.equal(y1, y2)
        for a, b in zip(r1, r2):
            assert torch.equal(a, b)
