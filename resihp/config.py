"""Closed-schema training configuration and fail-stop schedule.

The schema is a strict superset of the reference's (``resihp/config.py:49-136``): every
reference ``train.json`` and ``failures.json`` loads here unchanged and means the same
run (GPT-2 blocks, FP32, vocabulary 256, sequence 16, the reference AdamW settings).
The extra fields describe the Llama-style models and the bf16 B200 path:

==========================  ===========================================================
``arch``                    ``"gpt2"`` (reference blocks) or ``"llama"``
``vocab_size``/``seq_len``  token stream shape (reference run constants 256 / 16)
``ffn_dim``                 MLP width (GPT-2 default ``4 * model_dim``)
``num_kv_heads``            GQA key/value heads (default ``num_heads``)
``rope_theta``/``norm_eps`` Llama RoPE base and RMSNorm epsilon
``dtype``                   compute dtype: ``"fp32"`` or ``"bf16"`` (fp32 master + AdamW)
``tied_embeddings``         LM head shares the token embedding
``recompute``               activation recompute per transformer block
``sequence_parallel``       Megatron sequence parallelism inside TP groups
``init_std``                normal(0, std) init; ``null`` keeps torch's module defaults
``lr`` ``beta1`` ``beta2``  AdamW hyper-parameters (reference: 1e-3, 0.9, 0.999,
``adam_eps`` ``weight_decay``  1e-8, 0.01)
``checkpoint_every``        commit the logical checkpoint every N iterations
``memory_budget_bytes``     per-rank byte ceiling for the planner's memory gate
==========================  ===========================================================

One deliberate deviation: ``seed`` may be ``0`` (the reference demands a positive seed,
``resihp/config.py:98``, but the benchmark configuration names seed 0).

Failure files keep the reference contract exactly: only ``{"events": [...]}``, each
event only ``after_iteration`` (strictly increasing, positive) and ``failed_rank``
(unique, in range); any other key, e.g. a speed or heartbeat field, is rejected by name.
"""

from __future__ import annotations

from dataclasses import dataclass, fields
import json
from pathlib import Path
from typing import Any


class ConfigError(ValueError):
    """A training or failure configuration file is invalid."""


ARCHES = ("gpt2", "llama")
DTYPES = ("fp32", "bf16")


@dataclass(frozen=True)
class TrainConfig:
    model_dim: int
    num_layers: int
    num_heads: int
    batch_size: int
    micro_batch_size: int
    seed: int
    tp: int
    pp: int
    dp: int
    iterations: int
    memory_budget_bytes: int | None = None
    arch: str = "gpt2"
    vocab_size: int = 256
    seq_len: int = 16
    ffn_dim: int | None = None
    num_kv_heads: int | None = None
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    dtype: str = "fp32"
    tied_embeddings: bool = False
    recompute: bool = False
    sequence_parallel: bool = False
    init_std: float | None = None
    lr: float = 1e-3
    beta1: float = 0.9
    beta2: float = 0.999
    adam_eps: float = 1e-8
    weight_decay: float = 0.01
    checkpoint_every: int = 1

    @property
    def world_size(self) -> int:
        return self.tp * self.pp * self.dp

    @property
    def micro_batches(self) -> int:
        return self.batch_size // self.micro_batch_size

    @property
    def head_dim(self) -> int:
        return self.model_dim // self.num_heads

    @property
    def kv_heads(self) -> int:
        return self.num_heads if self.num_kv_heads is None else self.num_kv_heads

    @property
    def ffn(self) -> int:
        return 4 * self.model_dim if self.ffn_dim is None else self.ffn_dim


@dataclass(frozen=True)
class FailureEvent:
    after_iteration: int
    failed_rank: int


@dataclass(frozen=True)
class LoadedConfig:
    train: TrainConfig
    failures: tuple[FailureEvent, ...]


_REQUIRED = (
    "model_dim", "num_layers", "num_heads", "batch_size", "micro_batch_size",
    "seed", "tp", "pp", "dp", "iterations",
)
_OPTIONAL = {f.name for f in fields(TrainConfig)} - set(_REQUIRED)
_EVENT_KEYS = {"after_iteration", "failed_rank"}


def _load_json_object(path: Path, what: str) -> dict[str, Any]:
    try:
        value = json.loads(Path(path).read_text(encoding="utf-8"))
    except (OSError, json.JSONDecodeError) as error:
        raise ConfigError(f"cannot read {what} file {path}: {error}") from error
    if not isinstance(value, dict):
        raise ConfigError(f"{what} file must hold a JSON object: {path}")
    return value


def _int_field(raw: dict, key: str, what: str, *, floor: int = 1) -> int:
    value = raw.get(key)
    if type(value) is not int or value < floor:
        word = "positive" if floor == 1 else "non-negative"
        raise ConfigError(f"{what} field {key} must be a {word} integer")
    return value


def _float_field(raw: dict, key: str, what: str, *, positive: bool) -> float:
    value = raw[key]
    if type(value) not in (int, float) or (value <= 0 if positive else value < 0):
        raise ConfigError(f"{what} field {key} must be a {'positive' if positive else 'non-negative'} number")
    return float(value)


def _bool_field(raw: dict, key: str, what: str) -> bool:
    if type(raw[key]) is not bool:
        raise ConfigError(f"{what} field {key} must be true or false")
    return raw[key]


def parse_train(raw: dict[str, Any]) -> TrainConfig:
    """Validate a training-config object; see the module docstring for the schema."""
    what = "training config"
    missing = set(_REQUIRED) - raw.keys()
    if missing:
        raise ConfigError(f"{what} is missing fields: {sorted(missing)}")
    unknown = raw.keys() - set(_REQUIRED) - _OPTIONAL
    if unknown:
        raise ConfigError(f"{what} has unknown fields: {sorted(unknown)}")
    values: dict[str, Any] = {}
    for key in _REQUIRED:
        values[key] = _int_field(raw, key, what, floor=0 if key == "seed" else 1)
    for key in ("vocab_size", "seq_len", "checkpoint_every"):
        if key in raw:
            values[key] = _int_field(raw, key, what)
    for key in ("memory_budget_bytes", "ffn_dim", "num_kv_heads"):
        if raw.get(key) is not None:
            values[key] = _int_field(raw, key, what)
    for key in ("rope_theta", "norm_eps", "lr", "adam_eps"):
        if key in raw:
            values[key] = _float_field(raw, key, what, positive=True)
    for key in ("beta1", "beta2", "weight_decay"):
        if key in raw:
            values[key] = _float_field(raw, key, what, positive=False)
    if raw.get("init_std") is not None:
        values["init_std"] = _float_field(raw, "init_std", what, positive=True)
    for key in ("tied_embeddings", "recompute", "sequence_parallel"):
        if key in raw:
            values[key] = _bool_field(raw, key, what)
    if "arch" in raw:
        if raw["arch"] not in ARCHES:
            raise ConfigError(f"{what} field arch must be one of {ARCHES}")
        values["arch"] = raw["arch"]
    if "dtype" in raw:
        if raw["dtype"] not in DTYPES:
            raise ConfigError(f"{what} field dtype must be one of {DTYPES}")
        values["dtype"] = raw["dtype"]
    config = TrainConfig(**values)
    check_train(config)
    return config


def check_train(config: TrainConfig) -> None:
    """Cross-field constraints that every construction path must satisfy."""
    what = "training config"
    if config.model_dim % config.num_heads:
        raise ConfigError(f"{what} field model_dim must be divisible by num_heads")
    if config.batch_size % config.micro_batch_size:
        raise ConfigError(f"{what} field batch_size must be divisible by micro_batch_size")
    if config.num_heads % config.kv_heads:
        raise ConfigError(f"{what} field num_heads must be divisible by num_kv_heads")
    if config.arch == "gpt2" and config.kv_heads != config.num_heads:
        raise ConfigError(f"{what}: gpt2 blocks have no grouped-query attention")
    if config.arch == "gpt2" and config.sequence_parallel:
        raise ConfigError(f"{what}: sequence_parallel needs llama blocks (gpt2 blocks run the reference's "
                          "all-reduce tensor parallelism)")
    if config.seq_len < 2:
        raise ConfigError(f"{what} field seq_len must be at least 2 for next-token loss")
    if config.beta1 >= 1 or config.beta2 >= 1:
        raise ConfigError(f"{what}: AdamW betas must be below 1")


def parse_failures(raw: dict[str, Any], train: TrainConfig) -> tuple[FailureEvent, ...]:
    """Validate a failure schedule against ``train`` (reference ``config.py:109-136``)."""
    if set(raw) != {"events"} or not isinstance(raw.get("events"), list):
        raise ConfigError("failure config must hold exactly an events array")
    events: list[FailureEvent] = []
    last = 0
    seen: set[int] = set()
    for index, event in enumerate(raw["events"]):
        if not isinstance(event, dict):
            raise ConfigError(f"failure event {index} must be a JSON object")
        extra = event.keys() - _EVENT_KEYS
        if extra:
            raise ConfigError(f"failure event has forbidden field: {sorted(extra)[0]}")
        absent = _EVENT_KEYS - event.keys()
        if absent:
            raise ConfigError(f"failure event is missing fields: {sorted(absent)}")
        after = _int_field(event, "after_iteration", "failure event")
        rank = event["failed_rank"]
        if type(rank) is not int or not 0 <= rank < train.world_size:
            raise ConfigError(f"failure event failed_rank out of range: {rank}")
        if after <= last:
            raise ConfigError("failure event after_iteration must strictly increase")
        if rank in seen:
            raise ConfigError(f"failure event failed_rank repeated: {rank}")
        last = after
        seen.add(rank)
        events.append(FailureEvent(after, rank))
    return tuple(events)


def with_run_constants(config: TrainConfig, vocab_size: int | None = None,
                       sequence_length: int | None = None) -> TrainConfig:
    """``config`` with the token-stream shape a reference-style caller passes on its own
    (the reference keeps vocabulary and sequence length as run constants)."""
    from dataclasses import replace

    changes = {}
    if vocab_size is not None and vocab_size != config.vocab_size:
        changes["vocab_size"] = vocab_size
    if sequence_length is not None and sequence_length != config.seq_len:
        changes["seq_len"] = sequence_length
    return replace(config, **changes) if changes else config


def load_config(config_path: str | Path, failures_path: str | Path) -> LoadedConfig:
    train = parse_train(_load_json_object(Path(config_path), "training config"))
    failures = parse_failures(_load_json_object(Path(failures_path), "failure config"), train)
    return LoadedConfig(train=train, failures=failures)


def config_to_dict(config: TrainConfig) -> dict[str, Any]:
    """The JSON-serialisable form ``parse_train`` accepts back unchanged."""
    return {f.name: getattr(config, f.name) for f in fields(TrainConfig)}
