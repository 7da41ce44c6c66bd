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
