"""Tensor-parallel degree and membership selection (the only TP chooser).

Same decision rule as the reference (``resihp/planner/tp.py:137-198``): candidates are
the powers of two ``k`` with ``min_degree <= k <= |G'|``; a candidate survives when it
divides the model width, the head count and (when given) the vocabulary -- the token
embedding and LM head are vocab-parallel -- and, with a memory budget, when the
analytical memory model admits it. The **largest** survivor wins and its members are
the first ``k`` surviving ranks in ascending order. With Llama blocks a degree must also
divide the key/value head count and the MLP width, since both are column-sharded; for
the reference's GPT-2 blocks those two tests are implied by the first two.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, NamedTuple

from ..config import TrainConfig
from ..memory import memory_feasible
from ..validate import positive_int, unique_ranks


@dataclass(frozen=True)
class TPInfeasibleReason:
    code: str
    message: str
    active_ranks: tuple[int, ...]


class InfeasibleTP(ValueError):
    """No TP degree satisfies the constraints (stop code ``no_feasible_tp``)."""

    def __init__(self, reason: TPInfeasibleReason):
        super().__init__(reason.message)
        self.reason = reason


@dataclass(frozen=True)
class TPChoice:
    degree: int
    members: tuple[int, ...]


class _Budget(NamedTuple):
    sequence_length: int
    memory_budget: int
    in_flight_micro_batches: int


def power_of_two_degrees(limit: int, minimum: int) -> tuple[int, ...]:
    """Powers of two in ``[minimum, limit]``, ascending."""
    out = []
    k = 1
    while k <= limit:
        if k >= minimum:
            out.append(k)
        k <<= 1
    return tuple(out)


def degree_divides_model(config: TrainConfig, k: int, vocab_size: int | None) -> bool:
    """True when a stage can be sharded ``k`` ways at all (no memory question)."""
    if config.model_dim % k or config.num_heads % k:
        return False
    if config.kv_heads % k or config.ffn % k:
        return False
    return vocab_size is None or vocab_size % k == 0


def choose_tp(
    config: TrainConfig,
    *,
    active_ranks: Iterable[int],
    min_degree: int,
    stage_layers: int | None = None,
    micro_batches: int | None = None,
    sequence_length: int | None = None,
    vocab_size: int | None = None,
    memory_budget: int | None = None,
    in_flight_micro_batches: int | None = None,
) -> TPChoice:
    """The largest feasible TP degree for one stage's surviving ranks, and its members.

    ``active_ranks`` is already ``stage ranks - failed``; it is only sorted here.
    When ``memory_budget`` is set, ``sequence_length``, ``vocab_size`` and the stage's
    1F1B ``in_flight_micro_batches`` are required so the activation peak is never
    under-counted. Raises :class:`InfeasibleTP` when nothing survives.
    """
    min_degree = positive_int("min_degree", min_degree)
    ranks = unique_ranks("active_ranks", active_ranks)
    if config.model_dim % config.num_heads:
        raise ValueError("model_dim must be divisible by num_heads")
    layers = positive_int(
        "stage_layers", config.num_layers // config.pp if stage_layers is None else stage_layers
    )
    batches = positive_int(
        "micro_batches",
        config.batch_size // config.micro_batch_size if micro_batches is None else micro_batches,
    )
    vocab = None if vocab_size is None else positive_int("vocab_size", vocab_size)
    budget: _Budget | None = None
    if memory_budget is None:
        if sequence_length is not None:
            positive_int("sequence_length", sequence_length)
        if in_flight_micro_batches is not None:
            positive_int("in_flight_micro_batches", in_flight_micro_batches)
    else:
        limit = positive_int("memory_budget", memory_budget)
        if sequence_length is None or vocab is None or in_flight_micro_batches is None:
            raise ValueError(
                "sequence_length, vocab_size, and in_flight_micro_batches are required "
                "when memory_budget is set"
            )
        budget = _Budget(
            positive_int("sequence_length", sequence_length),
            limit,
            positive_int("in_flight_micro_batches", in_flight_micro_batches),
        )

    feasible = []
    for k in power_of_two_degrees(len(ranks), min_degree):
        if not degree_divides_model(config, k, vocab):
            continue
        if budget is not None and not memory_feasible(
            config,
            tp_degree=k,
            stage_layers=layers,
            micro_batches=batches,
            sequence_length=budget.sequence_length,
            vocab_size=vocab,
            memory_budget=budget.memory_budget,
            in_flight_micro_batches=budget.in_flight_micro_batches,
        ):
            continue
        feasible.append(k)
    if not feasible:
        raise InfeasibleTP(
            TPInfeasibleReason(
                "no_feasible_tp",
                "no TP degree satisfies active-rank, divisibility (heads, model "
                "dimension, vocabulary), and memory constraints",
                ranks,
            )
        )
    k = feasible[-1]
    return TPChoice(degree=k, members=ranks[:k])
