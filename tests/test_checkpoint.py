"""Checkpoint atomicity, validation and cross-compatibility with the reference."""

import json
import os
import subprocess
import sys

import pytest
import torch

from resihp.checkpoint import CheckpointError, load_anchor, load_checkpoint, save_checkpoint
from resihp.config import TrainConfig
from resihp.reference import ReferenceRun

C = TrainConfig(model_dim=16, num_layers=2, num_heads=4, batch_size=4, micro_batch_size=2, seed=3, tp=1, pp=1, dp=1,
                iterations=2, vocab_size=32, seq_len=8)
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def _saved(tmp_path, steps=1):
    run = ReferenceRun(C)
    for _ in range(steps):
        run.step()
    path = tmp_path / "ck.pt"
    save_checkpoint(path, C, run.full_state(), completed_steps=run.cursor, plan_version=2)
    return path, run


def test_roundtrip_and_validation(tmp_path):
    path, run = _saved(tmp_path)
    anchor, completed, version = load_checkpoint(path, C)
    assert completed == 1 and version == 2
    for name, (view, _d) in run.stage.local_shards().items():
        assert torch.equal(anchor[name]["param"], view)


def test_failed_replace_keeps_previous(tmp_path, monkeypatch):
    path, run = _saved(tmp_path)
    before = path.read_bytes()

    def boom(*a, **k):
        raise OSError("disk full")

    monkeypatch.setattr(os, "replace", boom)
    with pytest.raises(OSError):
        save_checkpoint(path, C, run.full_state(), completed_steps=5, plan_version=3)
    assert path.read_bytes() == before
    assert not (tmp_path / "ck.pt.tmp").exists()


def test_write_verification_catches_a_changed_byte_and_accepts_nan(tmp_path, monkeypatch):
    """The temp file is read back and compared with memory byte for byte: one flipped
    value aborts the write and keeps the previous file; NaNs (a diverged run) are kept
    as written and compare equal to themselves."""
    from resihp import checkpoint as ck

    path, run = _saved(tmp_path)
    before = path.read_bytes()
    real_load = ck._torch_load

    def flipped(p, mmap=False):
        payload = real_load(p, mmap)
        t = payload["params"]["lm_head.weight"]
        t.view(-1)[7] = t.view(-1)[7] + 1.0
        return payload

    monkeypatch.setattr(ck, "_torch_load", flipped)
    with pytest.raises(CheckpointError, match="write verification failed"):
        save_checkpoint(path, C, run.full_state(), completed_steps=5, plan_version=3)
    assert path.read_bytes() == before and not (tmp_path / "ck.pt.tmp").exists()
    monkeypatch.setattr(ck, "_torch_load", real_load)

    full = run.full_state()
    full["lm_head.weight"]["param"].view(-1)[3] = float("nan")
    save_checkpoint(path, C, full, completed_steps=1, plan_version=3)
    anchor, _ = load_anchor(path)
    assert torch.isnan(anchor["lm_head.weight"]["param"].view(-1)[3])


def test_each_corruption_is_its_own_root_cause(tmp_path):
    path, _ = _saved(tmp_path)
    payload = torch.load(path, weights_only=False)
    cases = {
        "format": dict(payload, format_version=9),
        "identity": dict(payload, identity=dict(payload["identity"], seed=4)),
        "missing": dict(payload, params={k: v for k, v in list(payload["params"].items())[1:]}),
        "cursor": dict(payload, completed_steps=7),
        "digest": dict(payload, params={**payload["params"], "final_norm.weight": payload["params"]["final_norm.weight"] + 1}),
    }
    messages = {"format": "format", "identity": "identity", "missing": "missing", "cursor": "cursor", "digest": "digest"}
    for key, bad in cases.items():
        torch.save(bad, path)
        with pytest.raises(CheckpointError, match=messages[key]):
            load_checkpoint(path, C)
    os.remove(path)
    with pytest.raises(CheckpointError, match="missing"):
        load_anchor(path)


@pytest.mark.reference
def test_reference_reads_our_checkpoint(tmp_path):
    path, run = _saved(tmp_path, steps=2)
    code = (
        "import sys, json; sys.path.insert(0, sys.argv[1])\n"
        "from resihp.checkpoint import load_anchor\n"
        "a, c = load_anchor(sys.argv[2]); print(json.dumps([c, sorted(a)]))\n"
    )
    out = subprocess.run([sys.executable, "-c", code, REF, str(path)], capture_output=True, text=True, check=True, cwd="/")
    completed, names = json.loads(out.stdout)
    assert completed == 2 and names == sorted(run.stage.logical_state_dict())


def test_background_writer_orders_writes_and_surfaces_errors(tmp_path):
    from resihp.checkpoint import CheckpointWriter

    run = ReferenceRun(C)
    writer = CheckpointWriter()
    path = tmp_path / "ck.pt"
    for step in range(1, 3):
        run.step()
        writer.submit(path, C, run.full_state(), completed_steps=step, plan_version=0)
    writer.flush()
    assert not writer.pending
    anchor, completed = load_anchor(path)
    assert completed == 2
    for name, (view, _d) in run.stage.local_shards().items():
        assert torch.equal(anchor[name]["param"], view)
    writer.submit(path, C, run.full_state(), completed_steps=3, plan_version=-1)
    with pytest.raises(CheckpointError, match="plan_version"):
        writer.flush()
    assert load_anchor(path)[1] == 2  # the failed write left the previous checkpoint in place
    writer.flush()  # the error is reported once


@pytest.mark.reference
def test_we_read_the_references_checkpoint(tmp_path):
    """A checkpoint the reference wrote (after two of its own steps) loads and validates
    here for the same configuration, names, step and values included."""
    path = tmp_path / "ref.pt"
    code = (
        "import sys, json; sys.path.insert(0, sys.argv[1])\n"
        "from resihp.config import TrainConfig\nfrom resihp.reference import ReferenceRun\n"
        "from resihp.checkpoint import save_checkpoint\n"
        "cfg = TrainConfig(model_dim=16, num_layers=2, num_heads=4, batch_size=4, micro_batch_size=2, seed=3,"
        " tp=1, pp=1, dp=1, iterations=2)\n"
        "run = ReferenceRun(cfg, vocab_size=32, sequence_length=8)\n"
        "run.step(); run.step()\n"
        "save_checkpoint(sys.argv[2], run, plan_version=1)\n"
        "print(json.dumps({k: v.tolist() for k, v in run.model.logical_state_dict().items()}))\n"
    )
    out = subprocess.run([sys.executable, "-c", code, REF, str(path)], capture_output=True, text=True, check=True,
                         cwd="/")
    theirs = json.loads(out.stdout)
    anchor, completed, version = load_checkpoint(path, C)
    assert completed == 2 and version == 1
    assert sorted(anchor) == sorted(theirs)
    for name, values in theirs.items():
        assert torch.equal(anchor[name]["param"], torch.tensor(values)), name
        assert int(anchor[name]["step"]) == 2


def test_reference_style_save_and_load_resume_a_run_bit_for_bit(tmp_path):
    """The reference's calls -- ``ReferenceRun(config, vocab_size=, sequence_length=)``,
    ``save_checkpoint(path, run, plan_version=)``, ``load_checkpoint(path, run)`` -- work
    here and a restored run continues exactly like the original."""
    base = TrainConfig(model_dim=16, num_layers=2, num_heads=4, batch_size=4, micro_batch_size=2, seed=3, tp=1,
                       pp=1, dp=1, iterations=4)
    run = ReferenceRun(base, vocab_size=32, sequence_length=8)
    first = [run.step() for _ in range(2)]
    assert run.config.vocab_size == 32 and run.sequence_length == 8
    assert first[0].tokens == tuple(tuple(r) for r in run.batches[0].tolist())
    path = save_checkpoint(tmp_path / "ck.pt", run, plan_version=1)
    other = ReferenceRun(base, vocab_size=32, sequence_length=8)
    assert load_checkpoint(path, other) == (2, 1) and other.cursor == 2
    a, b = run.step(), other.step()
    assert (a.loss, a.param_digest, a.optim_digest) == (b.loss, b.param_digest, b.optim_digest)
