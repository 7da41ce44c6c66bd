"""Deterministic data-parallel micro-batch assignment.

``assign(step, failure_signature, topology)`` is pure and keeps the reference's
semantics (``resihp/planner/dp.py:150-218``; the plan digest depends on them):

* a replica can take work only if no stage of its pipeline holds a failed rank;
* its capacity is the smallest stage capacity along its pipeline, where a stage's
  capacity is its own micro-batch bound (default: all of them) or 0 when the memory
  model rejects the stage at its 1F1B position; a replica of capacity 0 takes nothing;
* the step's micro-batches are apportioned over the capacity vector by the
  largest-remainder (Hamilton) method, equal remainders favouring the lower replica;
* micro-batch ids are consecutive ranges handed out replica by replica in replica
  order, and each micro-batch runs through every stage of its one replica.

The formulation here is vector-shaped: the topology is folded into one pipeline per
replica, every pipeline is reduced to one capacity (0 = excluded), and placements are
generated from the apportioned counts already in ``(micro_batch, stage_id)`` order.
"""

from __future__ import annotations

from collections import Counter
from dataclasses import dataclass
from itertools import groupby
from operator import attrgetter
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
        """Placements of each micro-batch (ascending ids), in placement order."""
        ordered = sorted(self.placements, key=attrgetter("micro_batch"))  # stable
        return {mb: tuple(group) for mb, group in groupby(ordered, key=attrgetter("micro_batch"))}

    @property
    def micro_batches_per_replica(self) -> dict[int, int]:
        """Distinct micro-batches each replica runs (ascending replica ids)."""
        runs = Counter(replica for replica, _ in {(p.replica_id, p.micro_batch) for p in self.placements})
        return dict(sorted(runs.items()))


@dataclass(frozen=True)
class DPInfeasibleReason:
    code: str
    message: str


class InfeasibleDP(ValueError):
    """No healthy replica can take the work (stop code ``no_feasible_dp_target``)."""

    def __init__(self, reason: DPInfeasibleReason):
        super().__init__(reason.message)
        self.reason = reason


def _validated(topology) -> DPTopology:
    """The topology, after every structural rule is checked (first violation raises)."""
    if not isinstance(topology, DPTopology):
        raise TypeError(f"expected a DPTopology, got {type(topology).__name__}")
    for name in ("micro_batches", "sequence_length", "vocab_size"):
        positive_int(name, getattr(topology, name))
    if topology.memory_budget is not None:
        positive_int("memory_budget", topology.memory_budget)
    if len(topology.stages) == 0:
        raise ValueError("a DP topology needs at least one stage")
    keys = [(s.replica_id, s.stage_id) for s in topology.stages]
    for stage in topology.stages:
        non_negative_int("replica_id", stage.replica_id)
        non_negative_int("stage_id", stage.stage_id)
        positive_int("stage_layers", stage.stage_layers)
        positive_int("tp_degree", stage.tp_degree)
        held = unique_ranks("stage ranks", stage.ranks)
        if len(held) != stage.tp_degree:
            raise ValueError(f"stage {stage.stage_id} of replica {stage.replica_id} lists {len(held)} ranks "
                             f"for TP degree {stage.tp_degree}")
        if keys.count((stage.replica_id, stage.stage_id)) > 1:
            raise ValueError(f"stage {stage.stage_id} of replica {stage.replica_id} appears more than once")
        if stage.capacity is not None:
            positive_int("capacity", stage.capacity)
    return topology


def stage_capacity(topology: DPTopology, stage: DPStage, *, index: int, num_stages: int) -> int:
    """Micro-batches ``stage`` can take at pipeline position ``index`` (0 = rejected by
    the memory model, replaying its 1F1B in-flight peak at that position)."""
    bound = topology.micro_batches if stage.capacity is None else stage.capacity
    if topology.memory_budget is None:
        return bound
    fits = memory_feasible(
        topology.config,
        tp_degree=stage.tp_degree,
        stage_layers=stage.stage_layers,
        micro_batches=topology.micro_batches,
        sequence_length=topology.sequence_length,
        vocab_size=topology.vocab_size,
        memory_budget=topology.memory_budget,
        in_flight_micro_batches=peak_in_flight(topology.micro_batches, stage_index=index, num_stages=num_stages),
    )
    return bound if fits else 0


def _pipelines(topology: DPTopology) -> list[tuple[DPStage, ...]]:
    """One stage tuple per replica, replicas ascending, stages ascending within each."""
    ordered = sorted(topology.stages, key=lambda s: (s.replica_id, s.stage_id))
    replicas = sorted({s.replica_id for s in ordered})
    return [tuple(s for s in ordered if s.replica_id == r) for r in replicas]


def _pipeline_capacity(topology: DPTopology, pipeline: tuple[DPStage, ...], dead: frozenset[int]) -> int:
    if not dead.isdisjoint(r for s in pipeline for r in s.ranks):
        return 0
    depth = len(pipeline)
    return min(stage_capacity(topology, s, index=i, num_stages=depth) for i, s in enumerate(pipeline))


def split_by_capacity(total: int, capacities: tuple[int, ...]) -> tuple[int, ...]:
    """Hamilton apportionment of ``total`` over ``capacities``: each entry gets the floor
    of its exact share, and the units left over go to the largest fractional parts
    (equal parts: lower index first). All-zero capacities get nothing."""
    weight = sum(capacities)
    if weight <= 0:
        return (0,) * len(capacities)
    exact = [divmod(total * c, weight) for c in capacities]  # (floor, remainder * weight)
    spare = total - sum(q for q, _ in exact)
    favoured = sorted(range(len(capacities)), key=lambda i: (-exact[i][1], i))[:spare]
    return tuple(q + (1 if i in favoured else 0) for i, (q, _) in enumerate(exact))


def assign(step: int, failure_signature: Iterable[int], active_topology: DPTopology) -> DPAssignment:
    """Place every micro-batch on exactly one healthy replica's whole pipeline."""
    step = non_negative_int("step", step)
    topology = _validated(active_topology)
    failures = unique_ranks("failure_signature", failure_signature)
    dead = frozenset(failures)

    pipelines = _pipelines(topology)
    capacity = [_pipeline_capacity(topology, p, dead) for p in pipelines]
    if max(capacity) <= 0:
        raise InfeasibleDP(DPInfeasibleReason(
            "no_feasible_dp_target",
            f"none of the {len(pipelines)} DP replicas can take micro-batches after failures {list(failures)}"))
    usable = [i for i, c in enumerate(capacity) if c > 0]
    counts = split_by_capacity(topology.micro_batches, tuple(capacity[i] for i in usable))

    placements: list[DPPlacement] = []
    next_id = 0
    for i, count in zip(usable, counts):
        for micro_batch in range(next_id, next_id + count):
            placements += [DPPlacement(micro_batch, s.stage_id, s.replica_id, s.ranks) for s in pipelines[i]]
        next_id += count
    # ids grow replica by replica and stages ascend inside each pipeline, so the list is
    # already in (micro_batch, stage_id) order
    return DPAssignment(step=step, failure_signature=failures, placements=tuple(placements))
