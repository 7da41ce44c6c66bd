"""The immutable, versioned execution plan: TP -> PP -> DP per replica.

A plan is a pure function of ``(config, step, version, cumulative failed ranks,
previous plan)``; ``previous`` supplies the old layout so that state routes describe
``previous -> current``. Communication ranks, TP shards and PP owners are read from the
current plan only -- never inferred from an older layout at run time.

This module reproduces the reference planner exactly (``resihp/plan.py:170-583``),
because the plan is the contract every rank must agree on and its canonical JSON /
SHA-256 digest is comparable across the two implementations:

* rank layout ``rank = (replica * PP + stage) * TP + tp_local``;
* per replica, each stage's survivors pick a TP degree (:func:`choose_tp`, memory-gated
  at the stage's old 1F1B position), then :func:`repartition_pp` moves layers; a
  replica that lost every stage is deferred, and if no replica is left the PP
  planner's own ``no_executable_pp`` is raised;
* a state group (one layer, or the ``embedding``/``head`` boundary group, which follow
  the replica's first/last executable stage) gets a :class:`StateRoute` exactly when
  its owning TP members change; the donor is the previous owner if it is fully alive,
  else the lowest-id peer replica whose owner is fully alive, else the checkpoint;
* the DP planner assigns micro-batches on the published layout, re-applying the memory
  gate, and :func:`assert_invariants` checks the result.
"""

from __future__ import annotations

from dataclasses import dataclass
from hashlib import sha256
import json
from typing import Iterable

from .config import TrainConfig
from .planner.dp import DPPlacement, DPStage, DPTopology, InfeasibleDP, assign
from .planner.pp import InfeasiblePP, balanced_layers, owner_ranges, peak_in_flight, repartition_pp
from .planner.tp import InfeasibleTP, choose_tp
from .validate import non_negative_int, unique_ranks

#: Persistent per-tensor state a route carries; ``grad`` is never persistent.
RECOVERED_STATES = ("param", "exp_avg", "exp_avg_sq", "step")
#: State groups owned by a replica's first / last executable stage.
BOUNDARY_GROUPS = ("embedding", "head")
DONOR_KINDS = frozenset({"prev_owner", "peer_replica", "checkpoint"})
RESHARD_METHODS = frozenset({"peer_copy", "gather_reshard", "checkpoint_restore"})


@dataclass(frozen=True)
class StagePlan:
    replica_id: int
    stage_id: int
    tp_degree: int
    tp_members: tuple[int, ...]
    layer_range: tuple[int, int]

    @property
    def stage_layers(self) -> int:
        return self.layer_range[1] - self.layer_range[0]


@dataclass(frozen=True)
class StateRoute:
    """How one state group of one replica reaches its new owners.

    ``layer`` is set for a layer group (``boundary == ""``); ``layer is None`` for a
    boundary group. ``donor_degree`` is 0 exactly for a checkpoint restore.
    """

    replica_id: int
    layer: int | None
    boundary: str
    target_ranks: tuple[int, ...]
    target_degree: int
    donor_kind: str
    donor_ranks: tuple[int, ...]
    donor_degree: int
    reshard: str
    states: tuple[str, ...] = RECOVERED_STATES


@dataclass(frozen=True)
class PlanInfeasibleReason:
    code: str
    message: str


class InfeasiblePlan(ValueError):
    def __init__(self, reason: PlanInfeasibleReason):
        super().__init__(reason.message)
        self.reason = reason


class PlanInvariantError(ValueError):
    """An ExecutionPlan violates a structural invariant."""


@dataclass(frozen=True)
class ExecutionPlan:
    version: int
    step: int
    config: TrainConfig
    failed_ranks: tuple[int, ...]
    active_ranks: tuple[int, ...]
    stages: tuple[StagePlan, ...]
    placements: tuple[DPPlacement, ...]
    state_routes: tuple[StateRoute, ...]

    def canonical(self) -> dict:
        """The normalised form the digest hashes (same key set as the reference)."""
        c = self.config
        return {
            "version": self.version,
            "step": self.step,
            "config": {
                "model_dim": c.model_dim, "num_layers": c.num_layers, "num_heads": c.num_heads,
                "batch_size": c.batch_size, "micro_batch_size": c.micro_batch_size,
                "tp": c.tp, "pp": c.pp, "dp": c.dp,
            },
            "failed_ranks": list(self.failed_ranks),
            "active_ranks": list(self.active_ranks),
            "stages": [
                [s.replica_id, s.stage_id, s.tp_degree, list(s.tp_members), list(s.layer_range)]
                for s in self.stages
            ],
            "placements": [
                [p.micro_batch, p.stage_id, p.replica_id, list(p.executor_ranks)] for p in self.placements
            ],
            "state_routes": [
                [
                    r.replica_id, r.layer, r.boundary, list(r.target_ranks), r.target_degree,
                    r.donor_kind, list(r.donor_ranks), r.donor_degree, r.reshard, list(r.states),
                ]
                for r in self.state_routes
            ],
        }

    @property
    def digest(self) -> str:
        text = json.dumps(self.canonical(), sort_keys=True, separators=(",", ":"))
        return sha256(text.encode("utf-8")).hexdigest()

    @property
    def live_ranks(self) -> tuple[int, ...]:
        dead = set(self.failed_ranks)
        return tuple(r for r in range(self.config.world_size) if r not in dead)


Layout = dict[int, dict[int, tuple[tuple[int, ...], tuple[int, int]]]]


def stage_domains(config: TrainConfig) -> dict[int, dict[int, tuple[int, ...]]]:
    """The pristine rank block of every (replica, stage)."""
    return {
        r: {
            s: tuple(range((r * config.pp + s) * config.tp, (r * config.pp + s + 1) * config.tp))
            for s in range(config.pp)
        }
        for r in range(config.dp)
    }


def _old_layout(config: TrainConfig, previous: ExecutionPlan | None) -> Layout:
    if previous is not None:
        layout: Layout = {}
        for s in previous.stages:
            layout.setdefault(s.replica_id, {})[s.stage_id] = (s.tp_members, s.layer_range)
        return layout
    domains = stage_domains(config)
    ranges = owner_ranges(tuple(len(x) for x in balanced_layers(config.num_layers, config.pp)))
    return {r: {s: (domains[r][s], ranges[s]) for s in range(config.pp)} for r in range(config.dp)}


def group_owner(stage_layout: dict, layer: int | None, boundary: str) -> tuple[int, ...]:
    """TP members owning a layer (by range) or a boundary group (first/last stage)."""
    if boundary:
        ids = sorted(stage_layout)
        return stage_layout[ids[0] if boundary == "embedding" else ids[-1]][0]
    for members, (lo, hi) in stage_layout.values():
        if lo <= layer < hi:
            return members
    raise AssertionError("layer is not owned by any stage in the layout")


def _repartition(old_layers, old_tp, new_tp):
    try:
        return repartition_pp(old_layers, old_tp, new_tp)
    except InfeasiblePP as error:
        raise InfeasiblePlan(PlanInfeasibleReason(error.reason.code, error.reason.message)) from error


def _route(old_layout: Layout, replica: int, layer, boundary: str, old_members, new_members, dead: set) -> StateRoute:
    def make(kind, donors, method):
        return StateRoute(
            replica_id=replica, layer=layer, boundary=boundary, target_ranks=new_members,
            target_degree=len(new_members), donor_kind=kind, donor_ranks=donors,
            donor_degree=len(donors), reshard=method,
        )

    if not dead.intersection(old_members):
        same = len(old_members) == len(new_members)
        return make("prev_owner", old_members, "peer_copy" if same else "gather_reshard")
    for peer in sorted(old_layout):
        if peer == replica:
            continue
        donors = group_owner(old_layout[peer], layer, boundary)
        if not dead.intersection(donors):
            return make("peer_replica", donors, "gather_reshard")
    return make("checkpoint", (), "checkpoint_restore")


def state_groups(num_layers: int) -> tuple[tuple[int | None, str], ...]:
    return tuple((layer, "") for layer in range(num_layers)) + tuple((None, b) for b in BOUNDARY_GROUPS)


def boundary_hops(plan: ExecutionPlan) -> tuple[tuple[int, ...], ...]:
    """Sorted union rank sets of every pipeline hop the assignment creates."""
    by_mb: dict[int, list[DPPlacement]] = {}
    for p in plan.placements:
        by_mb.setdefault(p.micro_batch, []).append(p)
    hops = set()
    for places in by_mb.values():
        chain = sorted(places, key=lambda p: p.stage_id)
        for up, down in zip(chain, chain[1:]):
            hops.add(tuple(sorted(set(up.executor_ranks) | set(down.executor_ranks))))
    return tuple(sorted(hops))


def build_plan(
    config: TrainConfig,
    *,
    step: int,
    version: int,
    failed_ranks: Iterable[int] = (),
    previous: ExecutionPlan | None = None,
    memory_budget: int | None = None,
    sequence_length: int = 1,
    vocab_size: int | None = None,
) -> ExecutionPlan:
    """Chain TP, PP and DP planning into one verified plan (see the module docstring)."""
    step = non_negative_int("step", step)
    version = non_negative_int("version", version)
    if previous is not None and not isinstance(previous, ExecutionPlan):
        raise TypeError("previous must be an ExecutionPlan or None")
    failed = unique_ranks("failed_ranks", failed_ranks)
    if failed and failed[-1] >= config.world_size:
        raise ValueError(f"failed_ranks contains an out-of-range rank: {failed[-1]}")
    dead = set(failed)
    micro_batches = config.batch_size // config.micro_batch_size
    domains = stage_domains(config)
    old = _old_layout(config, previous)

    stages: list[StagePlan] = []
    dp_stages: list[DPStage] = []
    routes: list[StateRoute] = []
    wiped: list[tuple[list[int], list[int], list[int]]] = []
    for replica in range(config.dp):
        old_layers = [0] * config.pp
        old_tp = [0] * config.pp
        for s, (members, (lo, hi)) in old.get(replica, {}).items():
            old_layers[s] = hi - lo
            old_tp[s] = len(members)
        # A stage's 1F1B position comes from the old pipeline (the new one needs the
        # degrees first); the DP gate re-checks the published layout below.
        old_live = [s for s in range(config.pp) if old_tp[s] > 0]

        chosen: dict[int, tuple[int, ...]] = {}
        new_tp = [0] * config.pp
        for s in range(config.pp):
            survivors = tuple(r for r in domains[replica][s] if r not in dead)
            if not survivors:
                continue
            try:
                pick = choose_tp(
                    config,
                    active_ranks=survivors,
                    min_degree=1,
                    stage_layers=max(1, old_layers[s]),
                    micro_batches=micro_batches,
                    sequence_length=sequence_length,
                    vocab_size=vocab_size,
                    memory_budget=memory_budget,
                    in_flight_micro_batches=peak_in_flight(
                        micro_batches, stage_index=old_live.index(s), num_stages=len(old_live)
                    ),
                )
            except InfeasibleTP as error:
                raise InfeasiblePlan(PlanInfeasibleReason(error.reason.code, error.reason.message)) from error
            chosen[s] = pick.members
            new_tp[s] = pick.degree

        if not any(new_tp):
            if any(old_tp):
                wiped.append((old_layers, old_tp, new_tp))
            continue

        pp_plan = _repartition(old_layers, old_tp, new_tp)
        new_layout = {}
        for s in range(config.pp):
            rng = pp_plan.layer_ranges[s]
            if rng is None:
                continue
            stages.append(StagePlan(replica, s, new_tp[s], chosen[s], rng))
            dp_stages.append(DPStage(replica, s, chosen[s], rng[1] - rng[0], new_tp[s]))
            new_layout[s] = (chosen[s], rng)
        # Stage-granular on purpose: any change of a group's owning members re-routes
        # the whole group to every new member.
        for layer, boundary in state_groups(config.num_layers):
            before = group_owner(old[replica], layer, boundary)
            after = group_owner(new_layout, layer, boundary)
            if before != after:
                routes.append(_route(old, replica, layer, boundary, before, after, dead))

    if not dp_stages:
        _repartition(*wiped[0])  # always raises no_executable_pp

    topology = DPTopology(
        config=config,
        stages=tuple(dp_stages),
        micro_batches=micro_batches,
        sequence_length=sequence_length,
        vocab_size=1 if vocab_size is None else vocab_size,
        memory_budget=memory_budget,
    )
    try:
        assignment = assign(step, failed, topology)
    except InfeasibleDP as error:
        raise InfeasiblePlan(PlanInfeasibleReason(error.reason.code, error.reason.message)) from error

    plan = ExecutionPlan(
        version=version,
        step=step,
        config=config,
        failed_ranks=failed,
        active_ranks=tuple(sorted({r for s in stages for r in s.tp_members})),
        stages=tuple(stages),
        placements=assignment.placements,
        state_routes=tuple(routes),
    )
    assert_invariants(plan, previous=previous)
    return plan


def assert_invariants(plan: ExecutionPlan, previous: ExecutionPlan | None = None) -> None:
    """Raise :class:`PlanInvariantError` unless every structural invariant holds.

    Single plan: active and failed ranks are disjoint; each rank sits in at most one
    stage; every replica's stages tile the model contiguously; every micro-batch runs
    each stage of exactly one replica exactly once; routes are well formed and never
    carry ``grad``. Across plans: the version strictly increases and failures only
    accumulate.
    """
    config = plan.config
    micro_batches = config.batch_size // config.micro_batch_size
    active = set(plan.active_ranks)
    failed = set(plan.failed_ranks)
    if len(active) != len(plan.active_ranks):
        raise PlanInvariantError("active_ranks contains duplicate ranks")
    if active & failed:
        raise PlanInvariantError("active and failed ranks overlap")
    seated = [r for s in plan.stages for r in s.tp_members]
    if len(seated) != len(set(seated)):
        raise PlanInvariantError("a rank is assigned to multiple stages")
    if set(seated) != active:
        raise PlanInvariantError("assigned ranks do not match active ranks")

    per_replica: dict[int, list[StagePlan]] = {}
    for s in plan.stages:
        if s.tp_degree != len(s.tp_members):
            raise PlanInvariantError("stage tp_degree does not match its member count")
        per_replica.setdefault(s.replica_id, []).append(s)
    live_stage_ids = {r: {s.stage_id for s in ss} for r, ss in per_replica.items()}
    for replica, ss in per_replica.items():
        cursor = 0
        for s in sorted(ss, key=lambda x: x.stage_id):
            if s.stage_layers < 1 or s.layer_range != (cursor, cursor + s.stage_layers):
                raise PlanInvariantError(f"replica {replica} layer ranges are not contiguous")
            cursor = s.layer_range[1]
        if cursor != config.num_layers:
            raise PlanInvariantError(f"replica {replica} layers do not cover the model")

    members = {(s.replica_id, s.stage_id): s.tp_members for s in plan.stages}
    by_mb: dict[int, list[DPPlacement]] = {}
    for p in plan.placements:
        if members.get((p.replica_id, p.stage_id)) != p.executor_ranks:
            raise PlanInvariantError("a placement executor does not match its stage TP members")
        by_mb.setdefault(p.micro_batch, []).append(p)
    if set(by_mb) != set(range(micro_batches)):
        raise PlanInvariantError("micro-batch coverage is incomplete")
    for mb, places in by_mb.items():
        replicas = {p.replica_id for p in places}
        if len(replicas) != 1:
            raise PlanInvariantError(f"micro-batch {mb} is split across replicas")
        ran = [p.stage_id for p in places]
        if len(ran) != len(set(ran)):
            raise PlanInvariantError(f"micro-batch {mb} runs a stage more than once")
        if set(ran) != live_stage_ids[replicas.pop()]:
            raise PlanInvariantError(f"micro-batch {mb} does not run its replica's stages exactly once")

    routed = set()
    for r in plan.state_routes:
        if r.donor_kind not in DONOR_KINDS or r.reshard not in RESHARD_METHODS:
            raise PlanInvariantError("state route has an unknown donor kind or reshard method")
        if (r.layer is None) == (r.boundary == ""):
            raise PlanInvariantError("state route must name exactly one layer or boundary")
        if r.boundary not in ("",) + BOUNDARY_GROUPS:
            raise PlanInvariantError("state route names an unknown boundary group")
        key = (r.replica_id, r.layer, r.boundary)
        if key in routed:
            raise PlanInvariantError("a state group is routed more than once")
        routed.add(key)
        if not r.target_ranks or set(r.target_ranks) - active:
            raise PlanInvariantError("state route target ranks are empty or not active")
        if r.target_degree != len(r.target_ranks):
            raise PlanInvariantError("state route target degree does not match its target ranks")
        if r.donor_degree != len(r.donor_ranks):
            raise PlanInvariantError("state route donor degree does not match its donor ranks")
        if not r.states:
            raise PlanInvariantError("state route migrates no state")
        if "grad" in r.states:
            raise PlanInvariantError("gradients are not persistent state and are never routed")
        if r.donor_kind == "checkpoint":
            if r.donor_ranks or r.reshard != "checkpoint_restore":
                raise PlanInvariantError("checkpoint route must have no donor ranks")
        elif not r.donor_ranks or set(r.donor_ranks) & failed:
            raise PlanInvariantError("state route donor ranks are empty or failed")

    if previous is not None:
        if plan.version <= previous.version:
            raise PlanInvariantError("plan version must strictly increase")
        if not set(previous.failed_ranks) <= failed:
            raise PlanInvariantError("failed ranks must grow monotonically")
