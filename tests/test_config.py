"""Closed-schema config and failure-schedule validation."""

import json

import pytest

from resihp.config import ConfigError, TrainConfig, config_to_dict, load_config, parse_train

BASE = {"model_dim": 128, "num_layers": 6, "num_heads": 8, "batch_size": 8, "micro_batch_size": 2, "seed": 1234,
        "tp": 2, "pp": 2, "dp": 2, "iterations": 8}


def _write(tmp_path, train, failures):
    a, b = tmp_path / "t.json", tmp_path / "f.json"
    a.write_text(json.dumps(train))
    b.write_text(json.dumps(failures))
    return a, b


def test_reference_files_load_unchanged(tmp_path):
    a, b = _write(tmp_path, dict(BASE, memory_budget_bytes=None), {"events": [{"after_iteration": 2, "failed_rank": 1}]})
    loaded = load_config(a, b)
    assert loaded.train.world_size == 8
    assert loaded.train.arch == "gpt2" and loaded.train.vocab_size == 256 and loaded.train.seq_len == 16
    assert loaded.failures[0].failed_rank == 1


@pytest.mark.parametrize("bad", [{"model_dim": 0}, {"tp": True}, {"seed": -1}, {"batch_size": 7}, {"num_heads": 7},
                                 {"surprise": 1}, {"arch": "bert"}, {"dtype": "fp8"}, {"num_kv_heads": 3, "arch": "llama"},
                                 {"sequence_parallel": True}])
def test_rejects_invalid_train(bad):
    with pytest.raises(ConfigError):
        parse_train(dict(BASE, **bad))


def test_seed_zero_is_accepted():
    assert parse_train(dict(BASE, seed=0)).seed == 0


def test_superset_roundtrip():
    cfg = parse_train(dict(BASE, arch="llama", vocab_size=1024, seq_len=128, ffn_dim=688, num_kv_heads=4,
                           dtype="bf16", tied_embeddings=True, recompute=True, sequence_parallel=True,
                           lr=3e-4, beta2=0.95, weight_decay=0.1))
    assert parse_train(config_to_dict(cfg)) == cfg


@pytest.mark.parametrize("events,msg", [
    ([{"after_iteration": 2, "failed_rank": 8}], "out of range"),
    ([{"after_iteration": 2, "failed_rank": 1}, {"after_iteration": 2, "failed_rank": 3}], "strictly increase"),
    ([{"after_iteration": 2, "failed_rank": 1}, {"after_iteration": 3, "failed_rank": 1}], "repeated"),
    ([{"after_iteration": 2, "failed_rank": 1, "speed": 0.5}], "forbidden field: speed"),
    ([{"after_iteration": 0, "failed_rank": 1}], "positive"),
])
def test_rejects_invalid_failures(tmp_path, events, msg):
    a, b = _write(tmp_path, BASE, {"events": events})
    with pytest.raises(ConfigError, match=msg):
        load_config(a, b)


def test_failures_need_only_events(tmp_path):
    a, b = _write(tmp_path, BASE, {"events": [], "heartbeat": 1})
    with pytest.raises(ConfigError):
        load_config(a, b)
