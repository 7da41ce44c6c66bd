"""Programmatic dependent launch keeps stream order: the same run with it on and off gives
bit-identical losses (runs late in the GPU tier).

A small Llama model in bf16 goes through the launched CLI (``python -m resihp.launch``)
twice, once with ``RESIHP_PDL=1`` (every step kernel scheduled during its predecessor's
tail, waiting on the device for it) and once with ``RESIHP_PDL=0`` (plain stream order):
on one GPU, and with two GPUs as two pipeline stages (NCCL send / receive between the
stages, stream-event ordering around them). Every kernel of the step is deterministic,
so a kernel that read a buffer before its producer had finished would change a loss.
No failure is scheduled.
"""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CONFIG = {
    "arch": "llama", "dtype": "bf16", "model_dim": 512, "num_layers": 2, "num_heads": 4, "ffn_dim": 1408,
    "vocab_size": 4096, "seq_len": 256, "batch_size": 4, "micro_batch_size": 2, "seed": 7,
    "tp": 1, "pp": 1, "dp": 1, "iterations": 3, "checkpoint_every": 100,
}


def _losses(workdir, pp, pdl):
    workdir.mkdir()
    cfg, fails = workdir / "train.json", workdir / "failures.json"
    cfg.write_text(json.dumps(dict(CONFIG, pp=pp)))
    fails.write_text(json.dumps({"events": []}))
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0", RESIHP_GROUP_TIMEOUT="120", RESIHP_PDL=pdl)
    out = subprocess.run([sys.executable, "-m", "resihp.launch", "--config", str(cfg), "--failures", str(fails),
                          "--timeout", "600"], cwd=workdir, env=env, capture_output=True, text=True, timeout=900)
    assert out.returncode == 0, (out.stdout[-3000:], out.stderr[-3000:])
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    return sorted((l["step"], l["rank"], l["loss"]) for l in lines if "step" in l and "loss" in l)


@pytest.mark.parametrize("pp", [1, 2])
def test_programmatic_launch_keeps_losses_bitwise(tmp_path, pp):
    if torch.cuda.device_count() < pp:
        pytest.skip(f"needs {pp} GPUs")
    on = _losses(tmp_path / "on", pp, "1")
    off = _losses(tmp_path / "off", pp, "0")
    assert [s for s, _, _ in on] == [1, 2, 3]
    assert on == off
