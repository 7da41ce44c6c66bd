"""The analytical memory model: exact reference formula, and the B200 regime's shape."""

import pytest

from resihp.config import TrainConfig
from resihp.memory import estimate_memory, memory_feasible

GPT2 = TrainConfig(model_dim=128, num_layers=4, num_heads=8, batch_size=8, micro_batch_size=2, seed=1, tp=2, pp=2,
                   dp=2, iterations=1)


def test_reference_formula_by_hand():
    m = estimate_memory(GPT2, tp_degree=2, stage_layers=2, micro_batches=4, sequence_length=8, vocab_size=32,
                        in_flight_micro_batches=2)
    d = 128
    layer = 12 * d * d + 4 * d
    assert m.sharded_parameters == 2 * layer * 4 // 2
    assert m.boundary_parameters == 2 * 32 * d * 4 // 2
    assert m.gradients == m.adam_exp_avg == m.adam_exp_avg_sq == m.sharded_parameters + m.boundary_parameters
    tokens = 2 * 2 * 8
    assert m.activation == tokens * d * 4 // 2 + tokens * d * 4


def test_budget_boundary_is_inclusive():
    kw = dict(tp_degree=1, stage_layers=1, micro_batches=2, sequence_length=4, vocab_size=16, in_flight_micro_batches=1)
    total = estimate_memory(GPT2, **kw).total
    assert memory_feasible(GPT2, memory_budget=total, **kw)
    assert not memory_feasible(GPT2, memory_budget=total - 1, **kw)


def test_llama_regime_recompute_and_sp_reduce_activations():
    base = dict(model_dim=2048, num_layers=24, num_heads=16, batch_size=64, micro_batch_size=2, seed=1, tp=2, pp=2,
                dp=2, iterations=1, arch="llama", vocab_size=32000, seq_len=2048, ffn_dim=5504, dtype="bf16")
    kw = dict(tp_degree=2, stage_layers=12, micro_batches=16, sequence_length=2048, vocab_size=32000,
              in_flight_micro_batches=2)
    plain = estimate_memory(TrainConfig(**base), **kw)
    sp = estimate_memory(TrainConfig(**base, sequence_parallel=True), **kw)
    rc = estimate_memory(TrainConfig(**base, recompute=True), **kw)
    assert sp.activation < plain.activation and rc.activation < plain.activation
    assert plain.sharded_parameters == sp.sharded_parameters
    # bf16 weights + fp32 master = 6 bytes per parameter; two fp32 gradient buffers (8 bytes)
    # and 4 bytes per moment
    params = (plain.sharded_parameters + plain.boundary_parameters) // 6
    assert plain.gradients == 8 * params and plain.adam_exp_avg == 4 * params
    # SP halves the block input and residual (d bf16 values per token and layer saved over
    # 2 micro-batches x 2048 tokens x 12 layers) and adds the fused TP workspace of one
    # micro-batch (two half-size publish slots, two partial buffers, one receive buffer)
    mb_tokens = 2 * 2048
    saved = 2 * mb_tokens * 12 * 2048 * 2
    workspace = (2 * mb_tokens // 2 + 3 * mb_tokens) * 2048 * 2
    assert sp.activation == plain.activation - saved + workspace


def test_rejects_overcount():
    with pytest.raises(ValueError):
        estimate_memory(GPT2, tp_degree=2, stage_layers=1, micro_batches=2, sequence_length=4, vocab_size=8,
                        in_flight_micro_batches=3)
