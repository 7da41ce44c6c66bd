"""The module-form decoder (``resihp.model``) against the training stage, on CPU in FP32.

The module is written from ``torch.nn`` layers and torch's scaled-dot-product
attention; the stage runs the framework's own op chain over a flat state. Same init,
same batch: the losses and every logical gradient must agree to FP32 rounding, and a
few ``torch.optim.AdamW`` steps of the module (built by ``resihp.reference.adamw``)
must track the stage's fused flat AdamW. Covers GPT-2 blocks (the reference's names),
Llama blocks with GQA, and tied embeddings; plus the reference-API helpers
(``next_token_loss``, ``logical_state_digest``, ``install_anchor``).
"""

import math

import pytest
import torch

from resihp.checkpoint import CheckpointError, install_anchor, load_anchor, save_checkpoint
from resihp.config import TrainConfig
from resihp.model import MLP_RATIO, ReferenceTransformer
from resihp.models.layout import model_specs
from resihp.reference import (ADAM_BETAS, LEARNING_RATE, ReferenceRun, adamw, logical_state_digest,
                              next_token_loss)
from resihp.verify import step_record

BASE = dict(model_dim=32, num_layers=3, num_heads=4, batch_size=4, micro_batch_size=2, seed=3, tp=1, pp=1, dp=1,
            iterations=3, vocab_size=64, seq_len=12)
CASES = {
    "gpt2": dict(BASE, arch="gpt2"),
    "llama-gqa": dict(BASE, arch="llama", num_kv_heads=2, ffn_dim=48, init_std=0.1),
    "llama-tied": dict(BASE, arch="llama", ffn_dim=48, tied_embeddings=True, init_std=0.1, rope_theta=500.0),
    "llama-recompute": dict(BASE, arch="llama", num_kv_heads=1, ffn_dim=40, init_std=0.1, recompute=True),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_parameter_names_are_the_logical_names(case):
    config = TrainConfig(**CASES[case])
    model = ReferenceTransformer(config)
    names = list(model.logical_state_dict())
    want = [s.name for s in model_specs(config)]
    assert sorted(names) == sorted(want)
    for s in model_specs(config):
        assert tuple(model.logical_state_dict()[s.name].shape) == s.shape
    assert model.layer_ids == tuple(range(config.num_layers))


@pytest.mark.parametrize("case", sorted(CASES))
def test_module_loss_and_gradients_match_the_stage(case):
    config = TrainConfig(**CASES[case])
    run = ReferenceRun(config)
    model = ReferenceTransformer(config)
    assert logical_state_digest(model) == logical_state_digest(run.stage)

    tokens = run.batches[0]
    record = step_record(run)  # the stage's loss and gradients for batch 0
    loss = model.loss(tokens)
    assert loss.item() == pytest.approx(record["loss"], rel=1e-5)
    assert next_token_loss(model(tokens), tokens, config.vocab_size).item() == pytest.approx(loss.item(), rel=1e-6)
    loss.backward()
    for name, param in model.logical_state_dict().items():
        torch.testing.assert_close(param.grad, record["grads"][name], rtol=1e-4, atol=1e-6, msg=name)


@pytest.mark.parametrize("case", ["gpt2", "llama-gqa"])
def test_module_training_tracks_the_stage(case):
    config = TrainConfig(**CASES[case])
    run = ReferenceRun(config)
    model = ReferenceTransformer(config)
    opt = adamw(model.parameters(), config)
    for i in range(3):
        tokens = run.batches[i]
        want = run.step()
        opt.zero_grad()
        loss = model.loss(tokens)
        loss.backward()
        opt.step()
        assert loss.item() == pytest.approx(want.loss, rel=1e-4)
    for name, param in model.logical_state_dict().items():
        torch.testing.assert_close(param.detach(), run.stage.logical_state_dict()[name].detach(), rtol=1e-4,
                                   atol=1e-5, msg=name)


def test_install_anchor_resumes_a_module_from_a_checkpoint(tmp_path):
    config = TrainConfig(**CASES["llama-gqa"])
    run = ReferenceRun(config)
    for _ in range(2):
        run.step()
    path = save_checkpoint(tmp_path / "ck.pt", config, run.full_state(), completed_steps=2)
    anchor, completed = load_anchor(path)
    model = ReferenceTransformer(config, init=False)
    opt = adamw(model.parameters(), config)
    install_anchor(model, opt, anchor)
    assert completed == 2 and logical_state_digest(model) == logical_state_digest(run.stage)
    for param in model.parameters():
        assert opt.state[param]["step"].item() == 2.0 and opt.state[param]["step"].device.type == "cpu"

    want = run.step()
    opt.zero_grad()
    loss = model.loss(run.batches[2])
    loss.backward()
    opt.step()
    assert loss.item() == pytest.approx(want.loss, rel=1e-5)
    for name, param in model.logical_state_dict().items():
        torch.testing.assert_close(param.detach(), run.stage.logical_state_dict()[name].detach(), rtol=1e-4,
                                   atol=1e-5, msg=name)

    partial = {k: v for k, v in anchor.items() if k != "final_norm.weight"}
    with pytest.raises(CheckpointError, match="final_norm.weight"):
        install_anchor(model, opt, partial)


def test_reference_signature_and_constants():
    config = TrainConfig(**CASES["gpt2"])
    model = ReferenceTransformer(config, vocab_size=32, sequence_length=8)
    assert model.vocab_size == 32 and model.sequence_length == 8
    assert model.logical_state_dict()["lm_head.weight"].shape == (32, 32)
    assert model.logical_state_dict()["layers.0.mlp.fc1.weight"].shape == (MLP_RATIO * 32, 32)
    with pytest.raises(ValueError, match="sequence length"):
        model(torch.zeros(2, 7, dtype=torch.long))
    opt = adamw(model.parameters())
    group = opt.param_groups[0]
    assert group["lr"] == LEARNING_RATE and group["betas"] == ADAM_BETAS


@pytest.mark.parametrize("case", sorted(CASES))
def test_parameter_counts_agree_with_the_memory_model(case):
    """The module, the layout table and the memory model count the same parameters
    (reference: ``tests/test_reference.py:110``, parameter count = memory model)."""
    from resihp.memory import layer_parameter_count
    from resihp.models.layout import layer_specs, parameter_count

    config = TrainConfig(**CASES[case])
    model = ReferenceTransformer(config)
    assert parameter_count(config) == sum(p.numel() for p in model.parameters())
    sharded, replicated = layer_parameter_count(config)
    block = sum(p.numel() for p in model.layers["0"].parameters())
    assert block == sharded + replicated == sum(math.prod(s.shape) for s in layer_specs(config, 0))
    if config.arch == "gpt2":
        d = config.model_dim
        assert block == 12 * d * d + 4 * d  # the reference's per-layer figure (FFN = 4d)
