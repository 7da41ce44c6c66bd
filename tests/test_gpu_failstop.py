"""Fail-stop recovery on GPUs with NCCL training groups (needs 4 GPUs).

Launches ``bench_recovery.py --small`` on 4 GPUs (TP2 x PP2, bf16, fused TP kernels over
peer memory, NCCL with NVLS disabled): rank 3 is SIGKILLed between steps, the survivors
replan onto 3 GPUs, move the lost state and keep training. No GPU is faulted: the kill
happens on the host at a safe point with nothing in flight.
"""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_failstop_on_four_gpus():
    if torch.cuda.device_count() < 4:
        pytest.skip("needs four GPUs")
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench_recovery.py"), "--gpus", "4", "--small", "--kills", "3:3",
         "--iterations", "6", "--timeout", "400"],
        capture_output=True, text=True, timeout=600, cwd=ROOT,
    )
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["launcher_rc"] == 0, line
    assert line["launch"]["killed_ranks"] == [3]
    ev = line["events"][0]
    assert ev["recovered"] and ev["plan_version"] == 1


def test_failstop_peer_replica_on_four_gpus():
    """TP1 x PP2 x DP2: the lost stage's state comes from the peer replica over NVLink."""
    if torch.cuda.device_count() < 4:
        pytest.skip("needs four GPUs")
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench_recovery.py"), "--gpus", "4", "--layout", "1,2,2", "--small",
         "--kills", "3:3", "--iterations", "6", "--timeout", "400"],
        capture_output=True, text=True, timeout=600, cwd=ROOT,
    )
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["launcher_rc"] == 0, line
    assert line["launch"]["killed_ranks"] == [3]
    ev = line["events"][0]
    assert ev["recovered"] and ev["plan_version"] == 1
    assert line["steps_seen"][-1] == 6
