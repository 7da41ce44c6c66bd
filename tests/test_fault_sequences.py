"""Random failure sequences through the planner: invariants and state coverage.

Thousands of seeded scenarios (random TP/PP/DP, model shape, micro-batching, memory
budget, and a random order of fail-stops) are replayed plan by plan (reference:
``tests/test_fault_sequences.py`` drives LCG-generated sequences the same way). Each
step either yields a plan or a stop with one of the six codes. Every plan must

* satisfy the structural invariants against its predecessor;
* route state only from live donors to active targets, never ``grad``;
* leave no gap for recovery: every tensor a rank owns under the new plan is either a
  shard it already held identically under the previous plan or the target of a route --
  exactly the condition under which :func:`resihp.recovery.recover` never raises
  "no state route covers";
* when no live rank holds some lost state (DP = 1), take it from the checkpoint.
"""

import pytest

import plan_scenarios
from resihp import config as config_mod
from resihp import plan as plan_mod
from resihp.control import STOP_CODES
from resihp.plan import assert_invariants
from resihp.recovery import route_names, routes_for, stage_layout, stage_of

COUNT = 1500


def _held(plan, rank):
    """``{name: (dim, index, degree)}`` this rank holds under ``plan``."""
    stage = stage_of(plan, rank)
    if stage is None:
        return {}
    idx = stage.tp_members.index(rank)
    return {n: (d, None if d is None else idx, None if d is None else stage.tp_degree)
            for n, d in stage_layout(plan, stage).items()}


def _check_transition(previous, plan):
    assert_invariants(plan, previous)
    active = set(plan.active_ranks)
    failed = set(plan.failed_ranks)
    for route in plan.state_routes:
        assert set(route.target_ranks) <= active
        if route.donor_kind != "checkpoint":
            assert not set(route.donor_ranks) & failed, route
    for rank in plan.active_ranks:
        before = _held(previous, rank)
        covered = set()
        for route in routes_for(plan, rank):
            covered |= set(route_names(plan.config, route))
        for name, layout in _held(plan, rank).items():
            assert name in covered or before.get(name) == layout, (rank, name, layout, before.get(name))


def _replay(scenario):
    config = config_mod.TrainConfig(**scenario["config"])
    kwargs = dict(memory_budget=scenario["budget"], sequence_length=scenario["seq"], vocab_size=scenario["vocab"])
    try:
        plan = plan_mod.build_plan(config, step=0, version=0, **kwargs)
    except plan_mod.InfeasiblePlan as stop:
        assert stop.reason.code in STOP_CODES
        return ["stop:" + stop.reason.code]
    trace = [plan.digest]
    failed = []
    for i, rank in enumerate(scenario["failures"]):
        failed.append(rank)
        try:
            nxt = plan_mod.build_plan(config, step=i + 1, version=plan.version + 1, failed_ranks=failed,
                                      previous=plan, **kwargs)
        except plan_mod.InfeasiblePlan as stop:
            assert stop.reason.code in STOP_CODES
            trace.append("stop:" + stop.reason.code)
            break
        _check_transition(plan, nxt)
        plan = nxt
        trace.append(plan.digest)
    return trace


@pytest.mark.parametrize("part", range(3))
def test_random_sequences_keep_invariants_and_cover_state(part):
    scenarios = plan_scenarios.scenarios(COUNT, seed=101 + part)
    traces = [_replay(s) for s in scenarios]
    plans = sum(1 for t in traces for x in t if not x.startswith("stop:"))
    stops = {x for t in traces for x in t if x.startswith("stop:")}
    assert plans > COUNT  # most scenarios survive at least one fail-stop
    assert stops, "the sequences should also exercise consistent stops"


def test_replay_is_deterministic():
    for s in plan_scenarios.scenarios(50, seed=5):
        assert _replay(s) == _replay(s)


def test_dp1_donor_exhaustion_uses_the_checkpoint():
    config = config_mod.TrainConfig(model_dim=64, num_layers=4, num_heads=4, batch_size=8, micro_batch_size=2, seed=1,
                                    tp=2, pp=2, dp=1, iterations=4)
    v0 = plan_mod.build_plan(config, step=0, version=0, vocab_size=64, sequence_length=8)
    v1 = plan_mod.build_plan(config, step=1, version=1, failed_ranks=(3,), previous=v0, vocab_size=64,
                             sequence_length=8)
    _check_transition(v0, v1)
    kinds = {r.donor_kind for r in v1.state_routes}
    assert kinds == {"checkpoint"}, kinds  # the dead rank's TP partner alone cannot rebuild its shards
