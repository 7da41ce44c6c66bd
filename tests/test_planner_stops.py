"""Planner stop codes reach every survivor identically (CPU/Gloo, real SIGKILLs).

A failure sequence that leaves no TP degree that fits the memory budget ends the job
with ``no_feasible_tp``; one that leaves no intact replica with capacity ends it with
``no_feasible_dp_target``. Every survivor raises the same :class:`ConsistentStop` at the
same safe point and leaves no process group behind (reference:
``tests/test_recovery.py:751-765``). ``no_executable_pp`` needs every rank of the world
dead, so it has no survivor to observe it; the pure planner tests cover it.
"""

import pytest

import dist_entries
from harness import assert_killed, read_results, run_ranks

CONFIG = dict(model_dim=32, num_layers=4, num_heads=4, batch_size=4, micro_batch_size=2, seed=2, tp=1, pp=2, dp=2,
              iterations=5, arch="llama", vocab_size=32, seq_len=8, ffn_dim=64, memory_budget_bytes=500_000)


@pytest.mark.slow
@pytest.mark.parametrize("schedule,code,survivors,at", [
    ({"1": 0, "2": 2}, "no_feasible_tp", [1, 3], 2),
    ({"1": 0, "2": 1, "3": 2}, "no_feasible_dp_target", [3], 3),
])
def test_planner_stop_is_consistent(schedule, code, survivors, at, tmp_path):
    codes = run_ranks(dist_entries.failstop_entry, 4, CONFIG, schedule, str(tmp_path))
    assert_killed(codes, list(schedule.values()), code)
    results = read_results(tmp_path, survivors)
    for r in results.values():
        assert r["stopped"] == code, r
        assert len(r["plans"]) == at  # one plan per fail-stop it recovered from, plus the initial one
