"""Post-failure layouts train like the single-process oracle (CPU/Gloo, real processes).

After a fail-stop the planner produces layouts no initial config does: a TP2 stage
feeding a TP1 stage (scatter/gather boundary), layers migrated between stages, replicas
with different TP degrees or PP layerings whose gradients meet through the logical
reduction path, tied embeddings held at two TP degrees. Each case trains the plan a
failure sequence leads to, from the seeded initialisation on the survivors, and must
match the oracle within the A2 band (reference: ``tests/test_parallel_pp.py:685-705``
and ``tests/test_parallel_dp.py:599-622`` cover the same layout families).
"""

import pytest
import torch

import dist_entries
from harness import read_results, run_ranks
from resihp.config import TrainConfig
from resihp.models.layout import shard_dims
from resihp.parallel.tp import local_slice
from test_distributed_numerics import BASE, STEPS, _oracle, assert_params_close

CASES = [
    (dict(tp=2, pp=2, dp=1), (3,)),                        # TP2 -> TP1 boundary, layer 2 migrates
    (dict(tp=1, pp=2, dp=2), (3,)),                        # replica 1 collapses to one 4-layer stage
    (dict(tp=2, pp=1, dp=2), (1,)),                        # replicas at TP1 and TP2
    (dict(tp=2, pp=2, dp=2, tied_embeddings=True), (5, 2)),  # two failures, tied pairs at mixed degrees
    (dict(tp=2, pp=1, dp=2, sequence_parallel=True), (1,)),  # SP replica (TP2) next to a TP1 replica
    (dict(tp=2, pp=2, dp=2, sequence_parallel=True, tied_embeddings=True), (5, 2)),  # all of it at once
    (dict(tp=1, pp=1, dp=4), (0,)),                        # 4 micro-batches over 3 replicas: a 2/1/1 split
    (dict(tp=4, pp=3, dp=1, num_kv_heads=4, num_layers=4), (4, 9, 6)),  # TP4 stages shrink twice, layers move
    (dict(tp=1, pp=3, dp=3, num_layers=4), (4, 5)),        # a replica loses two stages of three
]


@pytest.mark.slow
@pytest.mark.parametrize("layout,failed", CASES, ids=lambda c: str(c))
def test_post_failure_layout_matches_oracle(layout, failed, tmp_path):
    config = dict(BASE, **layout)
    world = config["tp"] * config["pp"] * config["dp"] - len(failed)
    codes = run_ranks(dist_entries.planned_entry, world, config, list(failed), STEPS, str(tmp_path))
    assert set(codes.values()) == {0}, codes
    results = read_results(tmp_path, range(world))
    ref_losses, ref_state = _oracle(config)
    by_replica = {}
    for r in results.values():
        if r["losses"][0] is not None:
            by_replica.setdefault(r["replica"], r["losses"])
    assert by_replica, "no rank reported a loss"
    for i, want in enumerate(ref_losses):
        got = sum(losses[i] for losses in by_replica.values())
        assert abs(got - want) <= 1e-4 * abs(want), (i, got, want)
    dims = shard_dims(TrainConfig(**config))
    seen = set()
    for r in results.values():
        for name, values in r.get("shards", {}).items():
            seen.add(name)
            want = local_slice(ref_state[name], dims[name], r["tp_rank"], r["tp_size"])
            assert_params_close(torch.tensor(values), want, lr=config.get("lr", 1e-3), steps=STEPS, name=name)
    assert seen == set(ref_state), sorted(set(ref_state) - seen)
