"""TP / PP / DP planner behaviour (decision rules, ties, errors)."""

import pytest

from resihp.config import TrainConfig
from resihp.planner.dp import DPStage, DPTopology, InfeasibleDP, assign, split_by_capacity
from resihp.planner.pp import (InfeasiblePP, balanced_layers, peak_in_flight, pipeline_phases, pipeline_schedule,
                               repartition_pp)
from resihp.planner.tp import InfeasibleTP, choose_tp

C = TrainConfig(model_dim=128, num_layers=6, num_heads=8, batch_size=8, micro_batch_size=2, seed=1, tp=4, pp=2,
                dp=2, iterations=1)


def test_tp_picks_largest_power_of_two_prefix():
    assert choose_tp(C, active_ranks=[7, 5, 6], min_degree=1).members == (5, 6)
    assert choose_tp(C, active_ranks=[3], min_degree=1).degree == 1
    with pytest.raises(InfeasibleTP):
        choose_tp(C, active_ranks=[1], min_degree=2)


def test_tp_respects_vocab_and_kv_heads():
    assert choose_tp(C, active_ranks=range(4), min_degree=1, vocab_size=6).degree == 2
    llama = TrainConfig(**{**C.__dict__, "arch": "llama", "num_kv_heads": 2, "ffn_dim": 344})
    assert choose_tp(llama, active_ranks=range(4), min_degree=1).degree == 2


def test_tp_rejects_bool_ranks():
    with pytest.raises(ValueError):
        choose_tp(C, active_ranks=[True], min_degree=1)


def test_1f1b_schedule_shape():
    assert pipeline_phases(4, stage_index=0, num_stages=2) == (1, 3)
    assert pipeline_schedule(3, stage_index=0, num_stages=3) == ("F", "F", "F", "B", "B", "B")
    assert pipeline_schedule(4, stage_index=1, num_stages=2) == ("F", "B") * 4
    assert peak_in_flight(8, stage_index=0, num_stages=4) == 4
    assert balanced_layers(5, 2) == ((0, 1, 2), (3, 4))


def test_repartition_paper_example_and_ties():
    plan = repartition_pp([3, 3], [2, 2], [1, 2])
    assert plan.stage_layers == (2, 4)
    assert plan.migrations == ((2, 0, 1),)
    dead = repartition_pp([3, 3], [2, 2], [0, 2])
    assert dead.stage_layers == (0, 6) and dead.embedding_owner == 1 and dead.lm_head_owner == 1
    with pytest.raises(InfeasiblePP):
        repartition_pp([3, 3], [2, 2], [0, 0])


def test_dp_split_and_reroute():
    assert split_by_capacity(5, (1, 1)) == (3, 2)
    assert split_by_capacity(4, (3, 1)) == (3, 1)
    stages = (DPStage(0, 0, (0,), 3, 1), DPStage(0, 1, (1,), 3, 1), DPStage(1, 0, (2,), 3, 1), DPStage(1, 1, (3,), 3, 1))
    topo = DPTopology(config=C, stages=stages, micro_batches=4)
    a = assign(0, [2], topo)
    assert {p.replica_id for p in a.placements} == {0}
    assert assign(0, [2], topo) == a
    with pytest.raises(InfeasibleDP):
        assign(0, [0, 2], topo)
