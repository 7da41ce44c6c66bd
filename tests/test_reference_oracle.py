"""The single-process oracle against the reference's own (CPU).

* the seeded token stream equals the reference's ``_token_stream`` batch for batch,
  including random access that rewinds the generator (``resihp/reference.py:97-103``);
* with the reference's architecture (GPT-2 blocks, FP32) and hyperparameters, this
  framework's oracle -- which runs the distributed stage code at TP degree 1 -- trains
  like the reference's ``ReferenceTransformer`` + ``torch.optim.AdamW``: same losses to
  reassociation precision, parameters within AdamW's conditioning;
* two oracle runs are bit-identical (loss and state digests);
* the module-form GPT-2 decoder (``resihp.model``) has the reference model's parameter
  names in the same order, its initial weights bit for bit, and its logits.

The reference is imported from ``baseline/_ref`` in a subprocess (both packages are
named ``resihp``); those tests skip when it is not installed (fail with
``RESIHP_REQUIRE_REFERENCE=1``).
"""

import json
import os
import subprocess
import sys

import pytest
import torch

from resihp.config import TrainConfig
from resihp.reference import ReferenceRun, token_stream

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
needs_ref = pytest.mark.reference

SHAPE = dict(model_dim=32, num_layers=2, num_heads=4, batch_size=4, micro_batch_size=2, seed=3, tp=1, pp=1, dp=1,
             iterations=4)
VOCAB, SEQ = 48, 8


def _in_reference(code, *args):
    out = subprocess.run([sys.executable, "-c", "import sys; sys.path.insert(0, sys.argv[1])\n" + code, REF, *args],
                         capture_output=True, text=True, check=True, cwd="/")
    return json.loads(out.stdout)


@needs_ref
def test_token_stream_matches_reference():
    theirs = _in_reference(
        "import json\nfrom resihp.reference import _token_stream\n"
        f"print(json.dumps([b.tolist() for b in _token_stream({VOCAB}, {SEQ}, 4, 5, 11)]))\n"
    )
    cfg = TrainConfig(**dict(SHAPE, seed=11), vocab_size=VOCAB, seq_len=SEQ)
    stream = token_stream(cfg)
    for i in (3, 0, 4, 1, 2):  # out of order: the stream rewinds its generator
        assert stream[i].tolist() == theirs[i], i


@needs_ref
def test_gpt2_oracle_trains_like_the_reference_transformer():
    theirs = _in_reference(
        "import json\nfrom resihp.config import TrainConfig\nfrom resihp.reference import ReferenceRun\n"
        f"run = ReferenceRun(TrainConfig(**{SHAPE!r}), vocab_size={VOCAB}, sequence_length={SEQ})\n"
        "losses = [run.step().loss for _ in range(4)]\n"
        "state = {k: v.tolist() for k, v in run.model.logical_state_dict().items()}\n"
        "print(json.dumps({'losses': losses, 'state': state}))\n"
    )
    ours = ReferenceRun(TrainConfig(**SHAPE, vocab_size=VOCAB, seq_len=SEQ))
    losses = [ours.step().loss for _ in range(4)]
    for got, want in zip(losses, theirs["losses"]):
        assert abs(got - want) <= 1e-5 * abs(want), (losses, theirs["losses"])
    state = {n: t for n, (t, _d) in ours.stage.local_shards().items()}
    assert set(state) == set(theirs["state"])
    for name, values in theirs["state"].items():
        want = torch.tensor(values)
        diff = (state[name] - want).abs()
        # AdamW's near-sign updates turn reassociation noise into at most 2 lr per step
        assert diff.max().item() <= 2 * 1e-3 * 4, name
        assert (diff > 1e-4 * want.abs() + 1e-5).float().mean().item() < 0.02, name


def test_oracle_is_repeatable():
    cfg = TrainConfig(**SHAPE, vocab_size=VOCAB, seq_len=SEQ, arch="llama", ffn_dim=64)
    a, b = ReferenceRun(cfg), ReferenceRun(cfg)
    for _ in range(3):
        ra, rb = a.step(), b.step()
        assert ra.loss == rb.loss and ra.param_digest == rb.param_digest and ra.optim_digest == rb.optim_digest


@needs_ref
def test_module_form_gpt2_equals_the_reference_transformer():
    """``resihp.model.ReferenceTransformer`` (GPT-2 blocks) built for the reference's
    config has the reference model's parameter names, the same initial weights bit for
    bit, and the same logits to FP32 rounding."""
    from resihp.model import ReferenceTransformer

    theirs = _in_reference(
        "import json, torch\nfrom resihp.config import TrainConfig\nfrom resihp.model import ReferenceTransformer\n"
        f"torch.manual_seed({SHAPE['seed']})\n"
        f"m = ReferenceTransformer(TrainConfig(**{SHAPE!r}), vocab_size={VOCAB}, sequence_length={SEQ})\n"
        f"tokens = torch.randint(0, {VOCAB}, (2, {SEQ}), generator=torch.Generator().manual_seed(5))\n"
        "print(json.dumps({'state': {k: v.tolist() for k, v in m.logical_state_dict().items()},\n"
        "                  'logits': m(tokens).tolist()}))\n"
    )
    ours = ReferenceTransformer(TrainConfig(**SHAPE, vocab_size=VOCAB, seq_len=SEQ))
    state = ours.logical_state_dict()
    assert list(state) == list(theirs["state"])
    for name, values in theirs["state"].items():
        assert torch.equal(state[name].detach(), torch.tensor(values)), name
    tokens = torch.randint(0, VOCAB, (2, SEQ), generator=torch.Generator().manual_seed(5))
    torch.testing.assert_close(ours(tokens).detach(), torch.tensor(theirs["logits"]), rtol=1e-5, atol=1e-5)
