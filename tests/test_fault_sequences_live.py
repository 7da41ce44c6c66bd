"""Seeded random fail-stop sequences through real processes (CPU/Gloo, 8 ranks).

Three kills at random iterations on TP2 x PP2 x DP2 (reference: ``tests/test_fault_sequences.py``
drives generated sequences through real ranks the same way). For each sequence: exactly
the scheduled ranks die; every survivor agrees on one plan per failure, equal to the
pure planner's; the data cursor never repeats or skips; each resume starts from a state
equal to the checkpoint (A1); and the first resumed iteration's loss equals the oracle
restarted from that checkpoint (A2).
"""

import os
import random

import pytest

import dist_entries
from harness import assert_killed, read_results, run_ranks
from resihp.checkpoint import load_anchor
from resihp.config import TrainConfig
from resihp.plan import build_plan
from resihp.verify import steps_from_anchor

CONFIG = dict(model_dim=64, num_layers=6, num_heads=4, batch_size=8, micro_batch_size=2, seed=11, tp=2, pp=2, dp=2,
              iterations=7, arch="llama", vocab_size=64, seq_len=16, ffn_dim=96, num_kv_heads=2, init_std=0.05)


def _sequence(seed):
    rng = random.Random(seed)
    victims = rng.sample(range(8), 3)
    iterations = sorted(rng.sample(range(1, 7), 3))
    return dict(zip(iterations, victims))


@pytest.mark.slow
@pytest.mark.parametrize("seed", [3, 6])
def test_random_sequence_recovers_consistently(seed, tmp_path):
    kills = _sequence(seed)
    config = TrainConfig(**CONFIG)
    codes = run_ranks(dist_entries.e2e_entry, 8, CONFIG, {str(k): v for k, v in kills.items()}, str(tmp_path))
    assert_killed(codes, sorted(kills.values()), f"sequence {seed}")
    survivors = [r for r in range(8) if r not in kills.values()]
    results = read_results(tmp_path, range(8))

    plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    digests, failed = [plan.digest], []
    for after, victim in sorted(kills.items()):
        failed.append(victim)
        plan = build_plan(config, step=after, version=plan.version + 1, failed_ranks=tuple(failed), previous=plan,
                          vocab_size=config.vocab_size, sequence_length=config.seq_len)
        digests.append(plan.digest)

    for r in survivors:
        res = results[r]
        assert res["stopped"] is None and res["plans"] == digests and res["initialized"] is False
        trained = [e for e in res["iterations"] if e["trained"]]
        assert [e["cursor"] for e in trained] == list(range(len(trained)))
        assert all(rec["a1"] in (True, None) for rec in res["recoveries"])

    for after in sorted(kills):
        anchor, completed = load_anchor(os.path.join(tmp_path, f"anchor_{after}.pt"))
        want = steps_from_anchor(config, anchor, start=completed, count=1)[0]["loss"]
        per_replica = {}
        for r in range(8):  # a rank killed after this iteration still reported it
            for e in results[r]["iterations"]:
                if e["iteration"] == after + 1 and e.get("loss") is not None:
                    per_replica.setdefault(e["replica"], e["loss"])
        got = sum(per_replica.values())
        assert abs(got - want) <= 1e-4 * abs(want), (after, got, want)


@pytest.mark.slow
@pytest.mark.parametrize("victim", [0, 1, 2, 3])
def test_losing_any_single_rank_recovers(victim, tmp_path):
    """TP2 x DP2 on four ranks, each rank killed in turn after iteration 2 -- including
    rank 0, the checkpoint writer and lowest rank (reference: the lose-every-rank family of
    ``tests/test_recovery.py``)."""
    run_config = dict(CONFIG, tp=2, pp=1, dp=2, num_layers=4, iterations=4)
    config = TrainConfig(**run_config)
    codes = run_ranks(dist_entries.e2e_entry, 4, run_config, {"2": victim}, str(tmp_path))
    assert_killed(codes, [victim], f"victim {victim}")
    survivors = [r for r in range(4) if r != victim]
    results = read_results(tmp_path, range(4))
    for r in survivors:
        res = results[r]
        assert res["stopped"] is None and len(res["plans"]) == 2 and res["initialized"] is False
        assert all(rec["a1"] in (True, None) for rec in res["recoveries"])
    anchor, completed = load_anchor(os.path.join(tmp_path, "anchor_2.pt"))
    want = steps_from_anchor(config, anchor, start=completed, count=2)
    for i, rec in enumerate(want):
        per_replica = {}
        for r in survivors:
            for e in results[r]["iterations"]:
                if e["iteration"] == 3 + i and e.get("loss") is not None:
                    per_replica.setdefault(e["replica"], e["loss"])
        got = sum(per_replica.values())
        assert abs(got - rec["loss"]) <= 1e-4 * abs(rec["loss"]), (victim, 3 + i, got, rec["loss"])


@pytest.mark.slow
def test_two_ranks_lost_at_one_boundary(tmp_path):
    """Two ranks of different replicas die after the same iteration: the survivors see
    both at one boundary, take one safe point for the pair (the plan the planner makes
    for both failures at once), and train on -- beyond the reference's schedule format,
    which names one rank per event."""
    kills = {"2": [2, 5]}
    config = TrainConfig(**CONFIG)
    codes = run_ranks(dist_entries.e2e_entry, 8, CONFIG, kills, str(tmp_path))
    assert_killed(codes, [2, 5], "pair")
    plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    after = build_plan(config, step=2, version=1, failed_ranks=(2, 5), previous=plan, vocab_size=config.vocab_size,
                       sequence_length=config.seq_len)
    results = read_results(tmp_path, [r for r in range(8) if r not in (2, 5)])
    for res in results.values():
        assert res["stopped"] is None and res["plans"] == [plan.digest, after.digest]
        assert all(rec["a1"] in (True, None) for rec in res["recoveries"])
        trained = [e for e in res["iterations"] if e["trained"]]
        assert [e["cursor"] for e in trained] == list(range(len(trained)))
    anchor, completed = load_anchor(os.path.join(tmp_path, "anchor_2.pt"))
    want = steps_from_anchor(config, anchor, start=completed, count=1)[0]["loss"]
    per_replica = {}
    for res in results.values():
        for e in res["iterations"]:
            if e["iteration"] == 3 and e.get("loss") is not None:
                per_replica.setdefault(e["replica"], e["loss"])
    assert abs(sum(per_replica.values()) - want) <= 1e-4 * abs(want)
