"""Principle A contracts on a resumed TP run (CPU/Gloo): A1 before resume, A2 after."""

import pytest

import dist_entries
from harness import read_results, run_ranks
from resihp import verify
from resihp.checkpoint import save_checkpoint
from resihp.config import TrainConfig
from resihp.reference import ReferenceRun

CONFIG = dict(model_dim=64, num_layers=2, num_heads=4, batch_size=4, micro_batch_size=2, seed=3, tp=2, pp=1, dp=1,
              iterations=4, arch="llama", vocab_size=64, seq_len=16, ffn_dim=96, num_kv_heads=2, init_std=0.05)


@pytest.mark.slow
def test_a1_and_a2_on_resumed_tp_run(tmp_path):
    oracle_cfg = TrainConfig(**dict(CONFIG, tp=1))
    run = ReferenceRun(oracle_cfg)
    run.step()
    run.step()
    anchor_path = tmp_path / "anchor.pt"
    save_checkpoint(anchor_path, oracle_cfg, run.full_state(), completed_steps=2, plan_version=0)
    codes = run_ranks(dist_entries.a2_entry, 2, CONFIG, str(anchor_path), 2, str(tmp_path))
    assert set(codes.values()) == {0}
    for r in read_results(tmp_path, [0, 1]).values():
        assert r["a1"] is True
        verify.assert_matches_reference(r["cmp"], label=f"rank {r['rank']}")


def test_reference_style_helpers():
    """The reference's verify helpers exist here with the same meaning: ``batch`` is the
    run's token stream, ``reference_steps`` the no-failure oracle from step 0, and the run
    constants it passes separately must agree with the config."""
    import pytest
    import torch

    from resihp import verify
    from resihp.config import TrainConfig
    from resihp.reference import ReferenceRun, token_stream

    cfg = TrainConfig(model_dim=32, num_layers=2, num_heads=4, batch_size=4, micro_batch_size=2, seed=3, tp=1, pp=1,
                      dp=1, iterations=2, arch="llama", vocab_size=48, seq_len=8, ffn_dim=64)
    assert torch.equal(verify.batch(cfg, 1, device="cpu"), token_stream(cfg)[1])
    with pytest.raises(ValueError):
        verify.batch(cfg, 0, device="cpu", vocab_size=256)
    recs = verify.reference_steps(cfg, count=2, vocab_size=48, sequence_length=8)
    run = ReferenceRun(cfg)
    assert [r["loss"] for r in recs] == [run.step().loss, run.step().loss]


def test_reference_call_forms():
    """``denominator(state)``, ``step_record(model, optimizer, tokens, vocab_size=)`` and
    ``initial_run(plan, rank=, vocab_size=, sequence_length=, tp_group=, ...)`` -- the
    reference's forms -- give what this package's own forms give."""
    import torch

    from resihp.model import ReferenceTransformer
    from resihp.plan import build_plan
    from resihp.recovery import initial_run
    from resihp.reference import adamw

    cfg = TrainConfig(model_dim=32, num_layers=2, num_heads=4, batch_size=4, micro_batch_size=2, seed=3, tp=1, pp=1,
                      dp=1, iterations=2, arch="llama", vocab_size=48, seq_len=8, ffn_dim=64, init_std=0.1)
    v = torch.rand(5, 3)
    assert torch.equal(verify.denominator({"exp_avg_sq": v, "step": torch.tensor(3.0)}),
                       verify.denominator(TrainConfig(**dict(CONFIG, beta2=0.999, adam_eps=1e-8)), v, 3))

    run = ReferenceRun(cfg)
    tokens = run.batches[0]
    ours = verify.step_record(run)
    model = ReferenceTransformer(cfg)
    theirs = verify.step_record(model, adamw(model.parameters(), cfg), tokens, vocab_size=48)
    assert set(theirs) == {"loss", "grads", "params", "moments"}
    assert abs(theirs["loss"] - ours["loss"]) <= 1e-5 * ours["loss"]
    for name, g in ours["grads"].items():
        torch.testing.assert_close(theirs["grads"][name], g, rtol=1e-4, atol=1e-6)

    plan = build_plan(cfg, step=0, version=0, vocab_size=48, sequence_length=8)
    first = initial_run(plan, rank=0, vocab_size=48, sequence_length=8, tp_group=None, executor_group=None,
                        boundary_groups={})
    assert first.step() == pytest.approx(ReferenceRun(cfg).step().loss, rel=1e-5)  # 2 micro-batches vs 1 pass
    with pytest.raises(ValueError, match="vocab_size=256"):
        initial_run(plan, rank=0, vocab_size=256, sequence_length=8, tp_group=None, executor_group=None,
                    boundary_groups={})
