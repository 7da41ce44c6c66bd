"""Restarting a stopped job from its checkpoint (``python -m resihp.launch --resume CK``).

A 4-iteration job leaves its checkpoint; a 7-iteration job restarted from it trains
iterations 5-7 only, and -- on the same TP2 x PP2 layout -- its losses equal an
uninterrupted 7-iteration run bit for bit (the state, the data cursor and the plan's
reduction orders are all the same). The checkpoint is topology-free, so the restart may
also run another layout (TP2 on two ranks here), which matches to reassociation
precision. Failure events at or before the checkpoint are in the past: only later ones
are scheduled. Real launcher, real processes, CPU/Gloo.
"""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BASE = dict(model_dim=32, num_layers=4, num_heads=4, batch_size=8, micro_batch_size=2, seed=5, tp=2, pp=2, dp=1,
            arch="llama", vocab_size=64, seq_len=8, ffn_dim=64, num_kv_heads=2, init_std=0.05)


def _launch(directory, iterations, *, resume=None, events=(), **layout):
    directory.mkdir()
    cfg, fails = directory / "train.json", directory / "failures.json"
    cfg.write_text(json.dumps(dict(BASE, iterations=iterations, **layout)))
    fails.write_text(json.dumps({"events": [{"after_iteration": a, "failed_rank": r} for a, r in events]}))
    cmd = [sys.executable, "-m", "resihp.launch", "--config", str(cfg), "--failures", str(fails), "--timeout", "300"]
    if resume is not None:
        cmd += ["--resume", str(resume)]
    env = dict(os.environ, PYTHONPATH=ROOT, OMP_NUM_THREADS="1")
    out = subprocess.run(cmd, cwd=directory, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, (out.stdout[-3000:], out.stderr[-3000:])
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    losses = {}
    for line in lines:
        if "step" in line:
            losses.setdefault(line["step"], set()).add(line["loss"])
    return lines, {k: sorted(v) for k, v in sorted(losses.items())}


@pytest.mark.slow
def test_restart_from_checkpoint_continues_the_run(tmp_path):
    _launch(tmp_path / "first", 4)
    checkpoint = tmp_path / "first" / "checkpoint.pt"
    assert checkpoint.exists()

    _, whole = _launch(tmp_path / "whole", 7)
    lines, resumed = _launch(tmp_path / "resumed", 7, resume=checkpoint, events=[(2, 1), (5, 3)])
    assert sorted(resumed) == [5, 6, 7]
    assert all(l["resume"]["completed_steps"] == 4 for l in lines if "resume" in l)
    launch = [l["launch"] for l in lines if "launch" in l][0]
    assert launch["scheduled_kills"] == [3] and launch["killed_ranks"] == [3]  # the kill after iteration 2 is past
    assert resumed[5] == whole[5]  # bitwise: same state, cursor and layout
    acceptance = [l["acceptance"] for l in lines if "acceptance" in l]
    assert acceptance and all(a["trained_iterations"][0] == 5 for a in acceptance)

    _, other = _launch(tmp_path / "other", 7, resume=checkpoint, tp=2, pp=1, dp=1)
    for it in (5, 6, 7):
        got, want = other[it][0], whole[it][0]
        assert abs(got - want) <= 1e-4 * abs(want), (it, got, want)


@pytest.mark.slow
def test_restarted_job_rolls_back_to_its_restart_point(tmp_path):
    """The restart checkpoint becomes the job's own checkpoint: with ``checkpoint_every =
    3`` a kill after iteration 5 -- before the restarted job's first commit, with no peer
    replica -- rolls every survivor back to iteration 4 instead of stopping."""
    _launch(tmp_path / "first", 4)
    checkpoint = tmp_path / "first" / "checkpoint.pt"
    lines, losses = _launch(tmp_path / "again", 7, resume=checkpoint, events=[(5, 3)], checkpoint_every=3)
    recoveries = [l["recovery"] for l in lines if "recovery" in l]
    assert recoveries and all(r["resumed_from"] == 4 for r in recoveries)
    assert not [l for l in lines if "stopped" in l]
    assert sorted(losses) == [5, 6, 7]
