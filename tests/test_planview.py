"""``python -m resihp.planview``: the plans a schedule produces, previewed without a run.

The digests it prints are the ones the planner (and so every rank at every safe point)
produces for the same schedule; a schedule the planner cannot serve ends with the
consistent-stop line the job would end with; and the tool imports no torch.
"""

import json
import os
import subprocess
import sys

from resihp.config import TrainConfig, load_config
from resihp.plan import build_plan
from resihp.planview import plans

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cli(*args):
    out = subprocess.run([sys.executable, "-m", "resihp.planview", *args], capture_output=True, text=True, cwd=ROOT,
                         env=dict(os.environ, PYTHONPATH=ROOT), check=True)
    return [json.loads(l) for l in out.stdout.splitlines()]


def test_shipped_schedule_digests_match_the_planner():
    lines = _cli("--config", "configs/train.json", "--failures", "configs/failures.json")
    loaded = load_config(os.path.join(ROOT, "configs/train.json"), os.path.join(ROOT, "configs/failures.json"))
    c = loaded.train
    plan = build_plan(c, step=0, version=0, vocab_size=c.vocab_size, sequence_length=c.seq_len)
    want, failed = [plan.digest], []
    for e in loaded.failures:
        failed.append(e.failed_rank)
        plan = build_plan(c, step=e.after_iteration, version=plan.version + 1, failed_ranks=failed, previous=plan,
                          vocab_size=c.vocab_size, sequence_length=c.seq_len)
        want.append(plan.digest)
    assert [l["plan"]["digest"] for l in lines] == want
    assert [l["plan"]["version"] for l in lines] == list(range(6))
    first, last = lines[0]["plan"], lines[-1]["plan"]
    assert first["routes"] == {} and first["micro_batches"] == {"0": 2, "1": 2}
    assert lines[1]["plan"]["routes"] == {"gather_reshard": 4}
    # replica 1 is gone: replica 0 keeps its layout (nothing moves) and takes every micro-batch
    assert last["failed_ranks"] == [1, 4, 5, 6, 7] and last["routes"] == {} and last["micro_batches"] == {"0": 4}
    assert all(l["plan"]["memory"]["max_rank_bytes"] > 0 for l in lines)
    assert len(_cli("--config", "configs/train.json")) == 1  # no schedule: the initial plan only


def test_a_schedule_the_planner_cannot_serve_ends_with_its_stop_code():
    config = TrainConfig(model_dim=32, num_layers=4, num_heads=4, batch_size=4, micro_batch_size=2, seed=2, tp=1,
                         pp=2, dp=2, iterations=5, arch="llama", vocab_size=32, seq_len=8, ffn_dim=64,
                         memory_budget_bytes=500_000)

    class Event:
        def __init__(self, after, rank):
            self.after_iteration, self.failed_rank = after, rank

    lines = list(plans(config, [Event(1, 0), Event(2, 2), Event(3, 1)]))
    assert [("plan" in l) for l in lines] == [True, True, False]
    assert lines[-1]["stopped"] == "no_feasible_tp" and lines[-1]["after_iteration"] == 2


def test_the_tool_is_torch_free():
    code = "import sys, resihp.planview; print('torch' in sys.modules)"
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=ROOT, check=True)
    assert out.stdout.strip() == "False"
