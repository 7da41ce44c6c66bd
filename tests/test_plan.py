"""ExecutionPlan construction and its invariants (crafted corruptions are rejected)."""

from dataclasses import replace

import pytest

from resihp.config import TrainConfig
from resihp.plan import InfeasiblePlan, PlanInvariantError, assert_invariants, boundary_hops, build_plan

C = TrainConfig(model_dim=128, num_layers=4, num_heads=8, batch_size=8, micro_batch_size=2, seed=1, tp=2, pp=2,
                dp=2, iterations=6)


def test_initial_plan_topology_and_stability():
    p = build_plan(C, step=0, version=1)
    assert p.active_ranks == tuple(range(8)) and p.state_routes == ()
    assert p.digest == build_plan(C, step=0, version=1).digest
    assert boundary_hops(p) == ((0, 1, 2, 3), (4, 5, 6, 7))


def test_failure_routes_and_donor_priority():
    v0 = build_plan(C, step=0, version=0)
    v1 = build_plan(C, step=2, version=1, failed_ranks=[1], previous=v0)
    kinds = {r.donor_kind for r in v1.state_routes}
    assert kinds <= {"prev_owner", "peer_replica"}
    assert all("grad" not in r.states for r in v1.state_routes)
    both = build_plan(C, step=2, version=1, failed_ranks=[1, 5], previous=v0)
    assert any(r.donor_kind == "checkpoint" for r in both.state_routes)


def test_whole_world_loss_stops_with_pp_code():
    v0 = build_plan(C, step=0, version=0)
    with pytest.raises(InfeasiblePlan) as err:
        build_plan(C, step=1, version=1, failed_ranks=range(8), previous=v0)
    assert err.value.reason.code == "no_executable_pp"


def test_memory_budget_stop_code():
    with pytest.raises(InfeasiblePlan) as err:
        build_plan(C, step=0, version=0, memory_budget=1000, vocab_size=32, sequence_length=8)
    assert err.value.reason.code == "no_feasible_tp"


@pytest.mark.parametrize("corrupt", [
    lambda p: replace(p, failed_ranks=(0,)),
    lambda p: replace(p, active_ranks=p.active_ranks + (0,)),
    lambda p: replace(p, placements=p.placements[:-1]),
    lambda p: replace(p, stages=(replace(p.stages[0], layer_range=(0, 1)),) + p.stages[1:]),
])
def test_invariants_reject_corruption(corrupt):
    p = build_plan(C, step=0, version=0)
    with pytest.raises(PlanInvariantError):
        assert_invariants(corrupt(p))


def test_cross_plan_invariants():
    v0 = build_plan(C, step=0, version=3)
    v1 = build_plan(C, step=1, version=4, failed_ranks=[2], previous=v0)
    with pytest.raises(PlanInvariantError):
        assert_invariants(replace(v1, version=3), previous=v0)
