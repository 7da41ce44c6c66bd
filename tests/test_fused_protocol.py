"""Race and deadlock checks of the fused kernels' protocols (model in ``fused_protocol``).

For the three TP ops (AG->GEMM, GEMM->RS, GEMM->AR), TP 2/4/8 and several grid sizes,
many random interleavings of four consecutive calls on every rank must finish without a
rank reading a block or tile of the wrong epoch, without deadlock, with every tile
computed exactly once per call, and with the host's claim bases (from the extension's
own host functions) equal to what the kernels claimed. A host whose per-call claim count
disagrees with the kernel's must be caught. The DP step is checked in both forms.

Deferred push releases (a copy agent keeping two or three partial-tile pushes in flight
and counting each one only after a later push is issued) are checked too: safe when the
agent pays every owed count before it waits on a peer, a deadlock when it carries them
into that wait.
"""

import pytest

from fused_protocol import ProtocolError, Simulation


@pytest.mark.parametrize("op", ["ag", "rs", "ar"])
@pytest.mark.parametrize("tp,grid", [(2, 3), (2, 8), (4, 5), (8, 7), (2, 20)])
def test_protocol_has_no_race_or_deadlock(op, tp, grid):
    for seed in range(5):
        sim = Simulation(op, tp=tp, rows_per_rank=256, n=512, grid=grid, epochs=4, seed=seed)
        assert sim.run() > 0


@pytest.mark.parametrize("op", ["rs", "ar"])
@pytest.mark.parametrize("tp,grid", [(2, 3), (4, 5), (8, 7)])
@pytest.mark.parametrize("depth", [2, 3])
def test_deferred_push_releases_paid_before_peer_waits(op, tp, grid, depth):
    for seed in range(3):
        assert Simulation(op, tp=tp, rows_per_rank=256, n=512, grid=grid, epochs=4, seed=seed,
                          push_depth=depth).run() > 0


def test_deferred_push_releases_carried_into_a_peer_wait_deadlock():
    # every copy agent ends its pushes still owing one count and then waits for the
    # peers' partials of its own tiles, which the peers' agents owe in the same way
    with pytest.raises(ProtocolError, match="deadlock"):
        Simulation("rs", tp=2, rows_per_rank=256, n=512, grid=3, epochs=4, seed=0, push_depth=2,
                   flush_before_wait=False).run()


def test_ag_without_the_gathered_copy():
    for seed in range(4):
        assert Simulation("ag", tp=4, rows_per_rank=256, n=512, grid=5, epochs=4, seed=seed,
                          keep_gathered=False).run() > 0


def test_a_host_counting_the_wrong_claims_is_caught():
    # a host that forgets the copy warps' one failing claim per CTA starts the next call's
    # claims in the middle of the items: units are skipped or repeated
    k = __import__("resihp.ops._ext", fromlist=["require"]).require()
    wrong = lambda: k.fused_copy_claims(1, 512, 512, 2, 4, 2, 3) - 8 * 3  # noqa: E731
    with pytest.raises(ProtocolError, match="race|deadlock|incomplete"):
        Simulation("ag", tp=2, rows_per_rank=256, n=512, grid=3, epochs=4, seed=0, copy_claims=wrong).run()


@pytest.mark.parametrize("push", [False, True], ids=["one-phase", "push"])
@pytest.mark.parametrize("dp,grid", [(2, 3), (3, 4), (4, 2), (8, 3)])
def test_dp_step_protocol_has_no_race_or_deadlock(dp, grid, push):
    from fused_protocol import DpSimulation

    for seed in range(8):
        assert DpSimulation(dp=dp, grid=grid, epochs=5, seed=seed, push=push).run() > 0
