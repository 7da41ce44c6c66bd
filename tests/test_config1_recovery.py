"""Llama-style decoder, CPU/Gloo, TP2 x PP2 x DP1, FP32, 20 steps.

Rank 3 is SIGKILLed after step 8; the survivors replan onto 3 ranks, reshard from the
last in-memory state / checkpoint, and continue. The losses of steps 9-20 must equal,
bit for bit, an uninterrupted run of the new plan started from the state the recovery
resumed from (the same checkpoint, the same data cursor).
"""

import pytest

import dist_entries
from harness import assert_killed, read_results, run_ranks

CONFIG = dict(
    model_dim=256, num_layers=4, num_heads=4, batch_size=8, micro_batch_size=2, seed=0, tp=2, pp=2, dp=1,
    iterations=20, arch="llama", vocab_size=1024, seq_len=128, ffn_dim=688, norm_eps=1e-5, rope_theta=10000.0,
    tied_embeddings=True, lr=1e-3, beta1=0.9, beta2=0.95, weight_decay=0.1, init_std=0.02,
)
KILL_AFTER = 8
VICTIM = 3


@pytest.mark.slow
def test_config1_failstop_matches_rerun_bitwise(tmp_path):
    fail_dir = tmp_path / "fail"
    fail_dir.mkdir()
    codes = run_ranks(dist_entries.failstop_entry, 4, CONFIG, {KILL_AFTER: VICTIM}, str(fail_dir))
    assert_killed(codes, [VICTIM], "config1")
    survivors = read_results(fail_dir, [0, 1, 2])
    assert all(r["stopped"] is None for r in survivors.values())
    plans = {tuple(r["plans"]) for r in survivors.values()}
    assert len(plans) == 1 and len(next(iter(plans))) == 2
    losses_after = {}
    for r in survivors.values():
        for it, loss in r["losses"].items():
            if int(it) > KILL_AFTER:
                losses_after[int(it)] = loss
    assert sorted(losses_after) == list(range(KILL_AFTER + 1, 21))

    rerun_dir = tmp_path / "rerun"
    rerun_dir.mkdir()
    anchor = fail_dir / f"anchor_{KILL_AFTER}.pt"
    codes = run_ranks(dist_entries.rerun_entry, 3, CONFIG, [VICTIM], KILL_AFTER, str(anchor), str(rerun_dir))
    assert set(codes.values()) == {0}
    rerun = {}
    for r in read_results(rerun_dir, [0, 1, 2]).values():
        assert r["plan"] == next(iter(plans))[1]
        rerun.update({int(k): v for k, v in r["losses"].items()})
    assert rerun == losses_after  # bitwise: identical floats
