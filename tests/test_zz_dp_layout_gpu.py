"""Pure data parallelism of the whole 1.3B model on two GPUs (runs last in the GPU tier).

``bench.py --gpus 2 --layout 1,1,2`` under torchrun: every GPU holds the full model
(one 29 GB flat-state region) and the fused DP all-reduce + AdamW kernel reads the
peer's whole gradient buffer each step. The bench line must report the layout it ran,
a positive throughput and no device error. Needs two GPUs; NVLS is off.
"""

import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_pure_dp_layout_on_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "bench.py"), "--gpus", "2", "--layout", "1,1,2",
           "--steps", "2", "--warmup", "1"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=900, cwd=ROOT, env=env)
    assert out.returncode == 0, out.stderr[-3000:]
    line = json.loads([l for l in out.stdout.splitlines() if l.startswith("{")][-1])
    assert line["config"]["parallelism"] == "tp1-pp1-dp2" and line["config"]["dp_comm"].startswith("fused")
    assert line["value"] > 0 and line["n_gpus"] == 2
