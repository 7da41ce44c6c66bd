"""The two recovery paths around the checkpoint cadence (CPU/Gloo, real SIGKILLs).

* **No checkpoint needed.** With a peer replica every lost shard survives on a live
  rank, so a run that never writes a checkpoint recovers exactly like one that writes
  one every iteration: after the fail-stop both continue with bit-identical losses.
* **Rollback.** Without a peer replica (DP = 1) the dead rank's shards come from the
  checkpoint. With ``checkpoint_every = 2`` a kill after iteration 3 finds a checkpoint of
  iteration 2: every survivor rolls back to it, re-runs iteration 3 onwards under the new
  plan, and matches, bit for bit, an uninterrupted run of the new plan from that
  checkpoint.
"""

import os

import pytest

import dist_entries
from harness import assert_killed, read_results, run_ranks

BASE = dict(model_dim=32, num_layers=4, num_heads=4, batch_size=8, micro_batch_size=2, seed=4, iterations=6,
            arch="llama", vocab_size=64, seq_len=8, ffn_dim=64, lr=1e-3, beta2=0.95)


def _losses_after(results, first):
    out = {}
    for r in results.values():
        for it, loss in r["losses"].items():
            if int(it) >= first:
                out.setdefault(int(it), set()).add(loss)
    return {it: sorted(v) for it, v in sorted(out.items())}


@pytest.mark.slow
def test_peer_replica_recovery_needs_no_checkpoint(tmp_path):
    runs = {}
    for every in (1, 1000):
        out = tmp_path / f"every{every}"
        out.mkdir()
        config = dict(BASE, tp=1, pp=2, dp=2, checkpoint_every=every)
        codes = run_ranks(dist_entries.failstop_entry, 4, config, {"2": 3}, str(out))
        assert_killed(codes, [3], f"checkpoint_every={every}")
        results = read_results(out, [0, 1, 2])
        assert all(r["stopped"] is None and r["recoveries"][0]["resumed_from"] == 2 for r in results.values())
        assert os.path.exists(out / "checkpoint.pt") == (every == 1)
        runs[every] = _losses_after(results, 3)
    assert runs[1] == runs[1000] and sorted(runs[1]) == [3, 4, 5, 6]


@pytest.mark.slow
def test_rollback_to_an_older_checkpoint_matches_a_rerun(tmp_path):
    config = dict(BASE, tp=2, pp=2, dp=1, checkpoint_every=2)
    codes = run_ranks(dist_entries.failstop_entry, 4, config, {"3": 3}, str(tmp_path))
    assert_killed(codes, [3], "rollback")
    results = read_results(tmp_path, [0, 1, 2])
    for r in results.values():
        assert r["stopped"] is None, r
        assert r["recoveries"][0]["after"] == 3 and r["recoveries"][0]["resumed_from"] == 2
    anchor = tmp_path / "anchor_3.pt"
    rerun_dir = tmp_path / "rerun"
    rerun_dir.mkdir()
    codes = run_ranks(dist_entries.rerun_entry, 3, config, [3], 3, str(anchor), str(rerun_dir))
    assert set(codes.values()) == {0}
    rerun = read_results(rerun_dir, [0, 1, 2])
    got = _losses_after(results, 3)
    want = {}
    for r in rerun.values():
        for it, loss in r["losses"].items():
            want.setdefault(int(it), set()).add(loss)
    assert got == {it: sorted(v) for it, v in sorted(want.items())} and sorted(got) == [3, 4, 5, 6]


@pytest.mark.slow
def test_group_churn_without_failure_is_transparent(tmp_path):
    """Every communicator torn down and rebuilt between iterations, the run rebuilt from
    its own state under the same plan: the losses equal an uninterrupted run bit for bit
    (reference: the ``dynamic_groups_pipeline`` gate of ``tests/test_combinations.py``)."""
    config = dict(BASE, tp=2, pp=2, dp=1, iterations=4)
    runs = {}
    for churn in (0, 2):
        out = tmp_path / f"churn{churn}"
        out.mkdir()
        codes = run_ranks(dist_entries.churn_entry, 4, config, churn, str(out))
        assert set(codes.values()) == {0}, codes
        runs[churn] = {r: v["losses"] for r, v in read_results(out, range(4)).items()}
    assert runs[0] == runs[2]


@pytest.mark.slow
def test_failure_before_the_first_checkpoint_rolls_back_to_the_initial_state(tmp_path):
    """``checkpoint_every = 3`` and a kill after iteration 2: no checkpoint exists yet and
    the dead rank's stage has no other holder. Every run of the config starts from the
    same seeded state, so the survivors roll back to it (cursor 0) instead of stopping,
    and re-run iterations 1-2 onwards under the new plan exactly like an uninterrupted
    run of that plan from the initial state."""
    from resihp.checkpoint import save_checkpoint
    from resihp.config import TrainConfig
    from resihp.models.init import initial_state

    config = dict(BASE, tp=1, pp=3, dp=1, checkpoint_every=3, iterations=5)
    codes = run_ranks(dist_entries.failstop_entry, 3, config, {"2": 2}, str(tmp_path))
    assert_killed(codes, [2], "early failure")
    results = read_results(tmp_path, [0, 1])
    for r in results.values():
        assert r["stopped"] is None, r
        assert r["recoveries"][0]["after"] == 2 and r["recoveries"][0]["resumed_from"] == 0
    anchor = tmp_path / "initial.pt"
    cfg = TrainConfig(**config)
    save_checkpoint(anchor, cfg, {n: {"param": t} for n, t in initial_state(cfg).items()}, completed_steps=0)
    rerun_dir = tmp_path / "rerun"
    rerun_dir.mkdir()
    codes = run_ranks(dist_entries.rerun_entry, 2, config, [2], 2, str(anchor), str(rerun_dir))
    assert set(codes.values()) == {0}
    want = {}
    for r in read_results(rerun_dir, [0, 1]).values():
        for it, loss in r["losses"].items():
            want.setdefault(int(it), set()).add(loss)
    assert _losses_after(results, 1) == {it: sorted(v) for it, v in sorted(want.items())}
