"""Race and deadlock checks of the fused TP kernels' protocol (model in ``fused_protocol``).

For both kernel variants, both ops, TP 2/4/8 and several grid sizes, many random
interleavings of four consecutive calls on every rank must finish without a rank
reading a row or tile of the wrong epoch and without deadlock. A host that advances its
counter bases by the wrong per-call step (the bug class met on a GPU once) must be
caught.
"""

import pytest

from fused_protocol import ProtocolError, Simulation


@pytest.mark.parametrize("variant", [0, 1])
@pytest.mark.parametrize("op", ["ag", "rs"])
@pytest.mark.parametrize("tp,grid", [(2, 3), (2, 8), (4, 5), (8, 7)])
def test_protocol_has_no_race_or_deadlock(op, variant, tp, grid):
    for seed in range(6):
        sim = Simulation(op, tp=tp, rows_per_rank=256, n=512, grid=grid, variant=variant, epochs=4, seed=seed)
        assert sim.run() > 0


def test_a_host_counting_the_wrong_copy_warps_is_caught():
    # variant 1 kernels have six copy warps per CTA; a host still counting four announces
    # an epoch before every warp published (a race), and after a few calls its targets
    # fall behind the counters so the announcement never comes (a deadlock)
    wrong = lambda grid: 4 * grid  # noqa: E731
    with pytest.raises(ProtocolError, match="race|deadlock"):
        Simulation("ag", tp=2, rows_per_rank=256, n=512, grid=3, variant=1, epochs=6, seed=0, host_step=wrong).run()


@pytest.mark.parametrize("dp,grid", [(2, 3), (3, 4), (4, 2), (8, 3)])
def test_dp_step_protocol_has_no_race_or_deadlock(dp, grid):
    from fused_protocol import DpSimulation

    for seed in range(8):
        assert DpSimulation(dp=dp, grid=grid, epochs=5, seed=seed).run() > 0
