"""Full 3-D fail-stop run: eight ranks, TP2 x PP2 x DP2, two real kills (CPU/Gloo).

Six layers, so halving a stage's TP degree also moves a layer across the stage boundary;
the kills hit rank 1 (replica 0) after iteration 2 and rank 5 (replica 1) after
iteration 4, so between the events the replicas run different layouts, and the second
event lands on the replica the first left untouched. The reference's end-to-end gate
(``tests/test_end_to_end.py:556-565``) checks the same families of invariants:

1. exactly the scheduled ranks die (exit -9) and stop recording after their iteration;
2. one new plan per failure, versions 0, 1, 2, the same digests on every rank, equal to
   the pure planner's for the same sequence;
3. the events reconfigure all three planes (a TP degree, a layer range, and the
   executors a (micro-batch, stage) pair is routed to all change);
4. every micro-batch runs every stage of exactly one replica, once, as the plan places
   it -- checked against what the ranks actually executed;
5. data is neither repeated nor skipped: the cursor advances by one every iteration;
6. before resuming, every placed rank's state equals the checkpoint (principle A1);
7. after resuming, each iteration's loss matches the single-process oracle restarted
   from the anchor of the last failure (principle A2), iterations 1-2 the plain oracle;
8. no process group survives the run, and none leaks across safe points: after each
   re-formation a rank holds no more groups than the initial plan needed.
"""

import os

import pytest

import dist_entries
from harness import assert_killed, read_results, run_ranks
from resihp.checkpoint import load_anchor
from resihp.config import TrainConfig
from resihp.plan import build_plan
from resihp.reference import ReferenceRun
from resihp.verify import steps_from_anchor

CONFIG = dict(model_dim=64, num_layers=6, num_heads=4, batch_size=8, micro_batch_size=2, seed=9, tp=2, pp=2, dp=2,
              iterations=6, arch="llama", vocab_size=64, seq_len=16, ffn_dim=96, num_kv_heads=2, init_std=0.05)
KILLS = {"2": 1, "4": 5}


def _plans(config):
    plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    plans, failed = [plan], []
    for after, rank in sorted((int(a), r) for a, r in KILLS.items()):
        failed.append(rank)
        plan = build_plan(config, step=after, version=plan.version + 1, failed_ranks=tuple(failed), previous=plan,
                          vocab_size=config.vocab_size, sequence_length=config.seq_len)
        plans.append(plan)
    return plans


@pytest.mark.slow
@pytest.mark.parametrize("sp", [False, True], ids=["tp", "tp-sp"])
def test_three_d_run_with_two_kills(tmp_path, sp):
    run_config = dict(CONFIG, sequence_parallel=sp)
    config = TrainConfig(**run_config)
    codes = run_ranks(dist_entries.e2e_entry, 8, run_config, KILLS, str(tmp_path))
    assert_killed(codes, [1, 5], "end-to-end")
    results = read_results(tmp_path, range(8))
    survivors = [r for r in range(8) if r not in (1, 5)]

    # 1. the dead stop recording at their kill
    assert [e["iteration"] for e in results[1]["iterations"]] == [1, 2]
    assert [e["iteration"] for e in results[5]["iterations"]] == [1, 2, 3, 4]

    # 2. one plan per failure, agreed and equal to the planner's
    plans = _plans(config)
    for r in survivors:
        assert results[r]["stopped"] is None
        assert results[r]["plans"] == [p.digest for p in plans]
        assert [x["version"] for x in results[r]["recoveries"]] == [1, 2]

    # 3. all three planes move
    def degrees(p):
        return {(s.replica_id, s.stage_id): s.tp_degree for s in p.stages}

    def ranges(p):
        return {(s.replica_id, s.stage_id): s.layer_range for s in p.stages}

    def routing(p):
        return {(x.micro_batch, x.stage_id): x.executor_ranks for x in p.placements}

    assert any(degrees(a) != degrees(b) for a, b in zip(plans, plans[1:]))
    assert any(ranges(a) != ranges(b) for a, b in zip(plans, plans[1:]))
    assert any(routing(a) != routing(b) for a, b in zip(plans, plans[1:]))

    # 4. every (micro-batch, stage) runs once, where the plan put it
    version_of = {}
    for r in survivors:
        for e in results[r]["iterations"]:
            version_of[e["iteration"]] = e["plan_version"]
    for it, version in version_of.items():
        executed = []
        for r in range(8):
            for e in results[r]["iterations"]:
                if e["iteration"] == it and e["trained"] and e.get("leader"):
                    executed += [(mb, e["stage"], e["replica"]) for mb in e["executed"]]
        want = sorted((p.micro_batch, p.stage_id, p.replica_id) for p in plans[version].placements)
        assert sorted(executed) == want, it

    # 5. the data cursor advances by one per iteration on every training rank
    for r in survivors:
        cursors = [e["cursor"] for e in results[r]["iterations"] if e["trained"]]
        assert cursors == list(range(len(cursors))) and len(cursors) == 6, (r, cursors)

    # 6. A1 before every resume
    for r in survivors:
        for rec in results[r]["recoveries"]:
            assert rec["a1"] in (True, None), (r, rec)
            assert rec["resumed_from"] == rec["after"]

    # 7. A2 after every resume: per-iteration loss (one reporter per replica) vs the oracle
    def loss_at(it):
        per_replica = {}
        for r in range(8):  # a rank killed after an iteration still reported that iteration
            for e in results[r]["iterations"]:
                if e["iteration"] == it and e.get("loss") is not None:
                    per_replica.setdefault(e["replica"], e["loss"])
        return sum(per_replica.values())

    oracle = ReferenceRun(TrainConfig(**dict(CONFIG, tp=1, pp=1, dp=1)))  # SP changes no math
    want = {1: oracle.step().loss, 2: oracle.step().loss}
    for after in (2, 4):
        anchor, completed = load_anchor(os.path.join(tmp_path, f"anchor_{after}.pt"))
        assert completed == after
        for i, rec in enumerate(steps_from_anchor(config, anchor, start=completed, count=2)):
            want[after + 1 + i] = rec["loss"]
    for it, w in want.items():
        got = loss_at(it)
        assert abs(got - w) <= 1e-4 * abs(w), (it, got, w)

    # 8. nothing left behind, nothing leaked across epochs
    for r in survivors:
        assert results[r]["initialized"] is False
        counts = results[r]["groups"]
        assert len(counts) == 3 and max(counts[1:]) <= counts[0], counts
