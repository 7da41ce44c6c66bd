"""Deterministic data-parallel micro-batch assignment.

``assign(step, failure_signature, topology)`` is a pure function with the reference's
semantics (``resihp/planner/dp.py:150-218``):

* a replica is a candidate only when no stage of its pipeline holds a failed rank;
* its capacity is the minimum over its stages of the memory gate -- the stage's own
  micro-batch capacity (default: all of them) or 0 when the memory model rejects the
  stage at its 1F1B position -- and a zero-capacity replica is dropped;
* micro-batches are split across candidates in proportion to capacity by largest
  remainder (ties to the lower candidate index), and numbered contiguously replica by
  replica, so each micro-batch flows through exactly one replica's whole pipeline.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable

from ..config import TrainConfig
from ..memory import memory_feasible
from ..validate import non_negative_int, positive_int, unique_ranks
from .pp import peak_in_flight


@dataclass(frozen=True)
class DPStage:
    """One PP stage of one DP replica."""

    replica_id: int
    stage_id: int
    ranks: tuple[int, ...]
    stage_layers: int
    tp_degree: int
    capacity: int | None = None


@dataclass(frozen=True)
class DPTopology:
    config: TrainConfig
    stages: tuple[DPStage, ...]
    micro_batches: int
    sequence_length: int = 1
    vocab_size: int = 1
    memory_budget: int | None = None


@dataclass(frozen=True)
class DPPlacement:
    """Who executes one (micro-batch, stage) pair."""

    micro_batch: int
    stage_id: int
    replica_id: int
    executor_ranks: tuple[int, ...]


@dataclass(frozen=True)
class DPAssignment:
    step: int
    failure_signature: tuple[int, ...]
    placements: tuple[DPPlacement, ...]

    @property
    def by_micro_batch(self) -> dict[int, tuple[DPPlacement, ...]]:
        out: dict[int, list[DPPlacement]] = {}
        for p in self.placements:
            out.setdefault(p.micro_batch, []).append(p)
        return {k: tuple(v) for k, v in out.items()}

    @property
    def micro_batches_per_replica(self) -> dict[int, int]:
        seen: dict[int, set[int]] = {}
        for p in self.placements:
            seen.setdefault(p.replica_id, set()).add(p.micro_batch)
        return {r: len(m) for r, m in seen.items()}


@dataclass(frozen=True)
class DPInfeasibleReason:
    code: str
    message: str


class InfeasibleDP(ValueError):
    """No healthy replica can take the work (stop code ``no_feasible_dp_target``)."""

    def __init__(self, reason: DPInfeasibleReason):
        super().__init__(reason.message)
        self.reason = reason


def _check(topology: DPTopology) -> None:
    if not isinstance(topology, DPTopology):
        raise TypeError("active_topology must be a DPTopology")
    positive_int("micro_batches", topology.micro_batches)
    positive_int("sequence_length", topology.sequence_length)
    positive_int("vocab_size", topology.vocab_size)
    if topology.memory_budget is not None:
        positive_int("memory_budget", topology.memory_budget)
    if not topology.stages:
        raise ValueError("active_topology must contain at least one stage")
    keys: set[tuple[int, int]] = set()
    for s in topology.stages:
        non_negative_int("replica_id", s.replica_id)
        non_negative_int("stage_id", s.stage_id)
        positive_int("stage_layers", s.stage_layers)
        positive_int("tp_degree", s.tp_degree)
        if len(unique_ranks("stage ranks", s.ranks)) != s.tp_degree:
            raise ValueError("stage ranks length must equal tp_degree")
        if (s.replica_id, s.stage_id) in keys:
            raise ValueError("active_topology contains duplicate replica/stage")
        keys.add((s.replica_id, s.stage_id))
        if s.capacity is not None:
            positive_int("capacity", s.capacity)


def stage_capacity(topology: DPTopology, stage: DPStage, *, index: int, num_stages: int) -> int:
    """Micro-batches ``stage`` can take at pipeline position ``index`` (0 = rejected)."""
    if topology.memory_budget is not None and not memory_feasible(
        topology.config,
        tp_degree=stage.tp_degree,
        stage_layers=stage.stage_layers,
        micro_batches=topology.micro_batches,
        sequence_length=topology.sequence_length,
        vocab_size=topology.vocab_size,
        memory_budget=topology.memory_budget,
        in_flight_micro_batches=peak_in_flight(topology.micro_batches, stage_index=index, num_stages=num_stages),
    ):
        return 0
    return topology.micro_batches if stage.capacity is None else stage.capacity


def split_by_capacity(total: int, capacities: tuple[int, ...]) -> tuple[int, ...]:
    """Largest-remainder split of ``total`` proportional to ``capacities``."""
    whole = sum(capacities)
    if whole <= 0:
        return tuple(0 for _ in capacities)
    shares = [total * c // whole for c in capacities]
    left = total - sum(shares)
    order = sorted(range(len(capacities)), key=lambda i: (-(total * capacities[i] % whole), i))
    for i in order[:left]:
        shares[i] += 1
    return tuple(shares)


def assign(step: int, failure_signature: Iterable[int], active_topology: DPTopology) -> DPAssignment:
    """Place every micro-batch on exactly one healthy replica's whole pipeline."""
    step = non_negative_int("step", step)
    _check(active_topology)
    failures = unique_ranks("failure_signature", failure_signature)
    dead = set(failures)

    replicas: dict[int, dict[int, DPStage]] = {}
    for s in active_topology.stages:
        replicas.setdefault(s.replica_id, {})[s.stage_id] = s

    candidates: list[tuple[tuple[DPStage, ...], int]] = []
    for replica in sorted(replicas):
        pipeline = tuple(replicas[replica][sid] for sid in sorted(replicas[replica]))
        if any(dead.intersection(s.ranks) for s in pipeline):
            continue
        capacity = min(
            stage_capacity(active_topology, s, index=i, num_stages=len(pipeline))
            for i, s in enumerate(pipeline)
        )
        if capacity > 0:
            candidates.append((pipeline, capacity))
    if not candidates:
        raise InfeasibleDP(
            DPInfeasibleReason("no_feasible_dp_target", "no healthy DP replica can accept the micro-batches")
        )

    counts = split_by_capacity(active_topology.micro_batches, tuple(c for _, c in candidates))
    placements = []
    mb = 0
    for (pipeline, _), count in zip(candidates, counts):
        for _ in range(count):
            placements.extend(DPPlacement(mb, s.stage_id, s.replica_id, s.ranks) for s in pipeline)
            mb += 1
    placements.sort(key=lambda p: (p.micro_batch, p.stage_id))
    return DPAssignment(step=step, failure_signature=failures, placements=tuple(placements))
