"""The launched CLI: ``python -m resihp.launch`` on the shipped 8-rank, 5-kill schedule.

Real processes, real SIGKILLs: the launcher must exit 0 (exactly the scheduled ranks
died of SIGKILL, every other rank exited cleanly), the survivors must have trained every
iteration and agree on one plan digest per fail-stop -- the digests the planner
produces for the same schedule (equal to the reference planner's).
"""

import json
import os
import subprocess
import sys

import pytest

from resihp.config import load_config
from resihp.plan import build_plan

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.slow
def test_shipped_schedule_end_to_end(tmp_path):
    cfg = os.path.join(ROOT, "configs", "train.json")
    fails = os.path.join(ROOT, "configs", "failures.json")
    env = dict(os.environ, PYTHONPATH=ROOT, OMP_NUM_THREADS="1")
    out = subprocess.run([sys.executable, "-m", "resihp.launch", "--config", cfg, "--failures", fails, "--timeout", "600"],
                         cwd=tmp_path, env=env, capture_output=True, text=True, timeout=900)
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    launch = [l["launch"] for l in lines if "launch" in l]
    assert out.returncode == 0, (out.stdout[-3000:], out.stderr[-3000:])
    assert launch and launch[0]["killed_ranks"] == [1, 4, 5, 6, 7]
    acceptance = [l["acceptance"] for l in lines if "acceptance" in l]
    assert sorted(a["rank"] for a in acceptance) == [0, 2, 3]

    loaded = load_config(cfg, fails)
    c = loaded.train
    plan = build_plan(c, step=0, version=0, vocab_size=c.vocab_size, sequence_length=c.seq_len)
    expected, failed = [plan.digest], []
    for e in loaded.failures:
        failed.append(e.failed_rank)
        plan = build_plan(c, step=e.after_iteration, version=plan.version + 1, failed_ranks=failed, previous=plan,
                          vocab_size=c.vocab_size, sequence_length=c.seq_len)
        expected.append(plan.digest)
    for a in acceptance:
        assert a["plan_versions"] == [0, 1, 2, 3, 4, 5]
        assert a["plan_digests"] == expected
        assert a["trained_iterations"] == list(range(1, 9))
        assert a["failed_ranks"] == [1, 4, 5, 6, 7] and a["world_members"] == [0, 2, 3]
    steps = [l for l in lines if "step" in l]
    assert {s["step"] for s in steps} == set(range(1, 9))
    assert sum(1 for l in lines if "recovery" in l) >= 5
