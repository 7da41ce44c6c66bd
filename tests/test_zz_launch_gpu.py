"""The launched CLI on eight GPUs: the shipped schedule under NCCL (runs last in the GPU tier).

``python -m resihp.launch --config configs/train.json --failures configs/failures.json``
with one worker per GPU and NCCL training groups (NVLS off), the reference's GPT-2 FP32
config on the plain-torch path: the launcher exits 0 with exactly the five scheduled
ranks SIGKILLed, and the survivors agree on the planner's digest stream (reference:
``tests/test_acceptance.py:297``). Kills happen on the host between iterations; no GPU
work is in flight.
"""

import json
import os
import subprocess
import sys

import pytest
import torch

from resihp.config import load_config
from resihp.plan import build_plan

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_shipped_schedule_on_eight_gpus(tmp_path):
    if torch.cuda.device_count() < 8:
        pytest.skip("needs eight GPUs")
    cfg = os.path.join(ROOT, "configs", "train.json")
    fails = os.path.join(ROOT, "configs", "failures.json")
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0", RESIHP_GROUP_TIMEOUT="120")
    out = subprocess.run([sys.executable, "-m", "resihp.launch", "--config", cfg, "--failures", fails, "--timeout", "600"],
                         cwd=tmp_path, env=env, capture_output=True, text=True, timeout=900)
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    assert out.returncode == 0, (out.stdout[-3000:], out.stderr[-3000:])
    launch = [l["launch"] for l in lines if "launch" in l]
    assert launch and launch[0]["killed_ranks"] == [1, 4, 5, 6, 7]
    acceptance = [l["acceptance"] for l in lines if "acceptance" in l]
    assert sorted(a["rank"] for a in acceptance) == [0, 2, 3]
    assert {a["device"] for a in acceptance} == {"cuda"} and {a["training_backend"] for a in acceptance} == {"nccl"}

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
        assert a["plan_digests"] == expected and a["trained_iterations"] == list(range(1, 9))
