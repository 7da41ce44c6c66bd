"""The single fail-stop recovery path, and a rank's training state under one plan.

Orchestration only: the planner's :class:`~resihp.plan.StateRoute` entries decide what
moves from which donor under which layout; :func:`recover` executes them (reference:
``resihp/recovery.py:373-468``). What is recovered is ``param``, ``exp_avg``,
``exp_avg_sq`` and ``step`` plus the data cursor; gradients are never persistent.

Transfers. On the CUDA bf16 path a peer route (``prev_owner`` / ``peer_replica``) is a
peer-to-peer pull: every rank publishes its flat-state region (a CUDA IPC handle plus
offsets) over the world group and each new owner copies the pieces of its new shards
straight from the donors' regions with one gather kernel, the re-partition to the new TP
degree expressed in the copy descriptors (:mod:`resihp.parallel.peer`). On the CPU /
FP32 path a peer route is one collective over the group of all live ranks: the donors
place their shards (every TP shard of the donor stage, a replicated tensor from its
first member only) into a full-size buffer, the buffer is summed, and each target keeps
its slice under the new degree. A ``checkpoint`` route is sliced straight from the
anchor. The reference moves the same state through a CPU object gather of the whole
model per donor degree.

Verification (principle A1): once installed, each rank's new shards are compared with
``torch.equal`` against the same slices of the checkpoint anchor; the agreed state
digest is the checkpoint's own content digest, identical on every rank. When the
checkpoint is older than the live state (``checkpoint_every > 1``) a plan that needs a
``checkpoint`` route rolls every rank back to the anchor; otherwise the live state is
kept and the digest is agreed over the ranks' local shard digests.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass, field
from hashlib import sha256

import torch
import torch.distributed as dist

from .checkpoint import CheckpointError, identity, read_payload, save_checkpoint, verify_digest
from .models.init import initial_stage_state
from .ops import _ext
from .parallel import peer
from .models.layout import group_specs, model_specs, stage_specs
from .parallel.dp import GradientReducer
from .parallel.pp import PipelineRuntime
from .parallel.reshard import ReshardError
from .parallel.tp import TensorParallelStage, local_slice
from .planner.dp import DPAssignment
from .reference import digest_tensors, token_stream

FIELDS = ("param", "exp_avg", "exp_avg_sq")


@dataclass
class TrainingGroups:
    """The process groups one rank holds under one plan (``None`` = not a member)."""

    world: object = None
    tp: object = None
    hops: dict = field(default_factory=dict)
    executor: object = None
    reduce: dict = field(default_factory=dict)
    live: object = None


# --- reading the plan -----------------------------------------------------------------


def stage_of(plan, rank):
    for s in plan.stages:
        if rank in s.tp_members:
            return s
    return None


def replica_stages(plan, replica):
    return sorted((s for s in plan.stages if s.replica_id == replica), key=lambda s: s.stage_id)


def stage_ends(plan, stage) -> tuple[bool, bool]:
    ends = replica_stages(plan, stage.replica_id)
    return stage.stage_id == ends[0].stage_id, stage.stage_id == ends[-1].stage_id


def stage_layout(plan, stage) -> dict[str, int | None]:
    first, last = stage_ends(plan, stage)
    return {s.name: s.shard_dim for s in stage_specs(plan.config, range(*stage.layer_range), first, last)}


def route_names(config, route) -> dict[str, int | None]:
    return {s.name: s.shard_dim for s in group_specs(config, route.layer, route.boundary)}


def routes_for(plan, rank) -> tuple:
    return tuple(r for r in plan.state_routes if rank in r.target_ranks)


def acquire_layout(plan, rank) -> dict[str, int | None]:
    out: dict[str, int | None] = {}
    for r in routes_for(plan, rank):
        out.update(route_names(plan.config, r))
    return out


def dp_assignment(plan) -> DPAssignment:
    return DPAssignment(step=plan.step, failure_signature=plan.failed_ranks, placements=plan.placements)


def _shape_of(config) -> dict[str, tuple]:
    return {s.name: s.shape for s in model_specs(config)}


# --- a rank's state under one plan -------------------------------------------------------


class PlannedRun:
    """This rank's stage and 1F1B runtime under ``plan``; ``cursor`` = completed steps."""

    def __init__(self, plan, *, rank, local_state, moments, groups: TrainingGroups, device, cursor, pin=False):
        sp = stage_of(plan, rank)
        first, last = stage_ends(plan, sp)
        self.plan = plan
        self.rank = rank
        self.device = torch.device("cpu") if device is None else torch.device(device)
        self.stage = TensorParallelStage(
            plan.config, layer_ids=range(*sp.layer_range), is_first=first, is_last=last,
            local_state=local_state, group=groups.tp, device=self.device, moments=moments,
        )
        reducer = GradientReducer(plan, rank, groups=groups.reduce, executor_group=groups.executor, replica_id=sp.replica_id)
        needs_reduce = bool(reducer.topology.dp_groups or reducer.topology.tied_groups or not reducer.topology.homogeneous
                            or self.stage.sp)
        if needs_reduce:
            reducer.attach(self.stage)
        self.runtime = PipelineRuntime(
            self.stage, rank=rank, replica_id=sp.replica_id, assignment=dp_assignment(plan),
            boundary_groups=groups.hops, reducer=reducer if needs_reduce else None,
        )
        self.batches = token_stream(plan.config, pin=pin and self.device.type == "cuda")
        self.cursor = cursor

    # the reference's run constants, carried by the config here
    @property
    def vocab_size(self) -> int:
        return self.plan.config.vocab_size

    @property
    def sequence_length(self) -> int:
        return self.plan.config.seq_len

    def step(self):
        loss = self.runtime.train_step(self.batches[self.cursor])
        self.cursor += 1
        return loss

    def local_state(self) -> dict:
        """``{name: {shard_index, shard_count, param, exp_avg, exp_avg_sq, step}}``."""
        st = self.stage
        step = torch.tensor(float(st.flat.step))
        out = {}
        for name, (view, _d) in st.local_shards().items():
            entry = {"shard_index": st.tp_rank, "shard_count": st.tp_size, "param": view}
            if st.flat.step > 0:
                entry.update(st.moment_views(name))
                entry["step"] = step
            out[name] = entry
        return out


def _reference_groups(plan, groups, *, vocab_size=None, sequence_length=None, world_group=None, tp_group=None,
                      executor_group=None, boundary_groups=None) -> TrainingGroups:
    """``groups``, or the :class:`TrainingGroups` the reference's keyword form names
    (``tp_group``, ``executor_group``, ``boundary_groups``, ``world_group``); the
    reference's run constants, when passed, must match the plan's config."""
    config = plan.config
    for name, given, have in (("vocab_size", vocab_size, config.vocab_size),
                              ("sequence_length", sequence_length, config.seq_len)):
        if given is not None and given != have:
            raise ValueError(f"{name}={given} does not match the config ({have})")
    if groups is not None:
        return groups
    return TrainingGroups(world=world_group, tp=tp_group, hops=dict(boundary_groups or {}), executor=executor_group)


def initial_run(plan, *, rank, groups: TrainingGroups | None = None, device=None, pin=False, **reference_form):
    """The run a rank starts with: the seeded initial weights cut to its stage and shard.

    ``reference_form``: the reference's keywords (``vocab_size``, ``sequence_length``,
    ``tp_group``, ``executor_group``, ``boundary_groups``) in place of ``groups``
    (reference ``resihp/recovery.py:262-305``).
    """
    groups = _reference_groups(plan, groups, **reference_form)
    sp = stage_of(plan, rank)
    if sp is None:
        return None
    first, last = stage_ends(plan, sp)
    full = initial_stage_state(plan.config, range(*sp.layer_range), first, last, device=device or "cpu")
    idx = sp.tp_members.index(rank)
    local = {
        s.name: local_slice(full[s.name], s.shard_dim, idx, sp.tp_degree)
        for s in stage_specs(plan.config, range(*sp.layer_range), first, last)
    }
    return PlannedRun(plan, rank=rank, local_state=local, moments={}, groups=groups, device=device, cursor=0, pin=pin)


# --- gathering the full logical state ---------------------------------------------------


def _canonical_holders(plan) -> dict[str, object]:
    """For each logical name, the one stage whose shards form its canonical copy."""
    out: dict[str, object] = {}
    for s in plan.stages:
        for name in stage_layout(plan, s):
            out.setdefault(name, s)
    return out


def gather_full_state(run, plan, *, group, dst: int | None, device, bucket_elems: int = 32 * 1024 * 1024,
                      staging=None):
    """Assemble ``{name: {param, exp_avg, exp_avg_sq, step}}`` on plan rank ``dst``.

    Every rank of ``group`` (the executor group) calls this; each element is contributed
    by exactly one rank of the name's canonical holder stage and summed, so the result is
    exact. ``dst=None`` makes every rank receive it. Returns ``None`` elsewhere.

    ``staging`` (a :class:`~resihp.checkpoint.CheckpointWriter`, CUDA only) makes the
    receiving rank copy each bucket into a reused page-locked buffer on a side stream
    instead of a synchronous ``.cpu()``; it then returns ``(state, event)`` with the event
    recorded after the last copy.
    """
    config = plan.config
    holders = _canonical_holders(plan)
    shapes = _shape_of(config)
    local = {} if run is None else run.local_state()
    step = 0 if run is None else run.stage.flat.step
    me = None if run is None else run.rank
    names = [s.name for s in model_specs(config)]
    out: dict[str, dict] = {n: {} for n in names}
    dst_group_rank = None if dst is None else plan.active_ranks.index(dst)
    want = dst is None or me == dst

    def numel(shape):
        n = 1
        for x in shape:
            n *= x
        return n

    buckets, cur, size = [], [], 0
    for n in names:
        cur.append(n)
        size += numel(shapes[n]) * len(FIELDS)
        if size >= bucket_elems:
            buckets.append(cur)
            cur, size = [], 0
    if cur:
        buckets.append(cur)

    deferred = staging is not None and want and torch.device(device).type == "cuda"
    side = staging.copy_stream(device) if deferred else None
    for index, bucket in enumerate(buckets):
        total = sum(numel(shapes[n]) for n in bucket) * len(FIELDS)
        buf = torch.zeros(total, dtype=torch.float32, device=device)
        off = 0
        for n in bucket:
            k = numel(shapes[n])
            holder = holders[n]
            entry = local.get(n)
            for f in FIELDS:
                if entry is not None and me in holder.tp_members and f in entry:
                    idx = holder.tp_members.index(me)
                    full = buf[off: off + k].view(shapes[n])
                    dim = dict(stage_layout(plan, holder))[n]
                    if dim is None:
                        if idx == 0:
                            full.copy_(entry[f])
                    else:
                        torch.chunk(full, holder.tp_degree, dim=dim)[idx].copy_(entry[f])
                off += k
        if dst is None:
            dist.all_reduce(buf, group=group)
        else:
            dist.reduce(buf, dst=dist.get_global_rank(group, dst_group_rank), group=group)
        if want:
            host = None
            if deferred:
                host = staging.pinned(index, total)
                side.wait_stream(torch.cuda.current_stream(device))
                with torch.cuda.stream(side):
                    host.copy_(buf, non_blocking=True)
                buf.record_stream(side)  # the allocator keeps buf until the copy is done
            off = 0
            for n in bucket:
                k = numel(shapes[n])
                for f in FIELDS:
                    view = buf[off: off + k].view(shapes[n])
                    out[n][f] = host[off: off + k].view(shapes[n]) if deferred else view.cpu()
                    off += k
    if not want:
        return None
    step_t = torch.tensor(float(step))
    full_state = {}
    for n in names:
        entry = {"param": out[n]["param"]}
        if step > 0:
            entry.update(exp_avg=out[n]["exp_avg"], exp_avg_sq=out[n]["exp_avg_sq"], step=step_t.clone())
        full_state[n] = entry
    if deferred:
        ready = torch.cuda.Event()
        ready.record(side)
        return full_state, ready
    return full_state


def commit_checkpoint(run, path, *, plan, groups: TrainingGroups | None = None, writer: bool,
                      cursor: int | None = None, device=None, background=None, group=None, **reference_form):
    """Safe-point step 2: gather every shard and atomically write the one checkpoint.

    ``background`` (a :class:`~resihp.checkpoint.CheckpointWriter`) moves the writer's
    file write to its thread; the gather itself is a collective and stays in line. The
    reference's form passes the executor group as ``group`` and the run constants, and
    lets the cursor default to the run's (reference ``resihp/recovery.py:340-370``).
    """
    groups = _reference_groups(plan, groups, executor_group=group, **reference_form)
    if cursor is None:
        cursor = 0 if run is None else run.cursor
    if groups.executor is None:
        return
    dst = plan.active_ranks[0]
    if writer and background is not None:
        background.flush()  # the previous write may still read the staging buffers
    staged = writer and background is not None and device is not None and torch.device(device).type == "cuda"
    full = gather_full_state(run, plan, group=groups.executor, dst=dst, device=device or "cpu",
                             staging=background if staged else None)
    if not writer:
        return
    ready = None
    if staged:
        full, ready = full
    if background is not None:
        background.submit(path, plan.config, full, completed_steps=cursor, plan_version=plan.version, ready=ready)
    else:
        save_checkpoint(path, plan.config, full, completed_steps=cursor, plan_version=plan.version)


def logical_digest(full) -> str:
    return digest_tensors(sorted((f"{n}.{k}", t) for n, fs in full.items() for k, t in fs.items()))


# --- the single recovery path ------------------------------------------------------------


def _route_transfer(config, route, local, rank, *, group, device):
    """Execute one peer route; returns this rank's new shards if it is a target."""
    specs = group_specs(config, route.layer, route.boundary)
    sizes = []
    for s in specs:
        n = 1
        for x in s.shape:
            n *= x
        sizes.append(n)
    per_field = sum(sizes)
    buf = torch.zeros(per_field * len(FIELDS) + 1, dtype=torch.float32, device=device)
    if rank in route.donor_ranks:
        idx = route.donor_ranks.index(rank)
        for fi, f in enumerate(FIELDS):
            off = fi * per_field
            for s, k in zip(specs, sizes):
                entry = local.get(s.name)
                if entry is None or f not in entry:
                    raise ReshardError(f"donor rank {rank} does not hold {s.name}.{f}")
                full = buf[off: off + k].view(s.shape)
                if s.shard_dim is None:
                    if idx == 0:
                        full.copy_(entry[f])
                else:
                    torch.chunk(full, route.donor_degree, dim=s.shard_dim)[idx].copy_(entry[f])
                off += k
        if idx == 0:
            buf[-1] = float(local[specs[0].name]["step"])
    dist.all_reduce(buf, group=group)
    if rank not in route.target_ranks:
        return {}
    t = route.target_ranks.index(rank)
    out = {}
    step = buf[-1].detach().cpu().clone()
    for s, k in zip(specs, sizes):
        out[s.name] = {}
    for fi, f in enumerate(FIELDS):
        off = fi * per_field
        for s, k in zip(specs, sizes):
            full = buf[off: off + k].view(s.shape)
            out[s.name][f] = local_slice(full, s.shard_dim, t, route.target_degree)
            off += k
    for s in specs:
        out[s.name]["step"] = step.clone()
    return out


def _anchor_slices(config, route, anchor, rank):
    t = route.target_ranks.index(rank)
    out = {}
    for s in group_specs(config, route.layer, route.boundary):
        entry = anchor.get(s.name)
        if entry is None:
            raise ReshardError(f"logical tensor {s.name} unavailable from peers and checkpoint")
        out[s.name] = {f: local_slice(entry[f], s.shard_dim, t, route.target_degree) for f in FIELDS if f in entry}
        if "step" in entry:
            out[s.name]["step"] = entry["step"].clone()
    return out


def _load_anchor(checkpoint_path):
    """``(anchor, completed_steps, digest)`` of a checkpoint, ``None`` if there is none."""
    from pathlib import Path

    if checkpoint_path is None or not Path(checkpoint_path).exists():
        return None
    payload = read_payload(checkpoint_path)
    verify_digest(payload)
    anchor = {}
    for name, param in payload["params"].items():
        entry = {"param": param}
        if name in payload["optim"]:
            entry.update(payload["optim"][name])
        anchor[name] = entry
    return anchor, payload["completed_steps"], payload["digest"]


class InitialAnchor(Mapping):
    """The seeded initial state as a checkpoint anchor (``{name: {"param"}}``, no moments,
    zero completed steps), built name by name as recovery asks for it.

    Every run of a config starts from this state, bit for bit on every rank, so a
    failure that comes before the first checkpoint commit rolls back to it instead of
    stopping: the iterations before the failure are re-run under the new plan.
    """

    def __init__(self, config, device=None):
        self.config = config
        # the initial state does not depend on the device it is drawn for; kept on the host
        self.device = torch.device("cpu") if device is None else torch.device(device)
        self.names = [s.name for s in model_specs(config)]
        self._known = frozenset(self.names)
        self.digest = sha256(("initial-state:" + repr(sorted(identity(config).items()))).encode("utf-8")).hexdigest()
        self._built: dict[str, dict] = {}

    def __getitem__(self, name):
        if name not in self._built:
            if name not in self._known:
                raise KeyError(name)
            from .models.init import initial_state

            # GPT-2 blocks are drawn from one generator in module order: build them all once
            wanted = None if self.config.arch == "gpt2" else [name]
            for n, t in initial_state(self.config, names=wanted).items():  # the same values on any device
                self._built.setdefault(n, {"param": t})
        return self._built[name]

    def __contains__(self, name):
        return name in self._known  # a membership test draws nothing

    def __iter__(self):
        return iter(self.names)

    def __len__(self):
        return len(self.names)


def state_fingerprint(run) -> str:
    """Cheap, deterministic fingerprint of one rank's shards (computed on its device)."""
    if run is None:
        return ""
    st = run.stage
    sums = []
    for buf in (st.flat.master, st.flat.exp_avg, st.flat.exp_avg_sq):
        b = buf.double()
        sums += [float(b.sum()), float(b.abs().sum()), float((b * b).sum())]
    return sha256(repr((st.flat.step, [f"{x:.17g}" for x in sums])).encode("utf-8")).hexdigest()


def _collective_recover(run, local, *, plan, rank, anchor, rollback, completed, groups, device, tdev, cursor, pin):
    """Peer routes as one collective each over the live group (CPU / FP32 path)."""
    config = plan.config
    stage = stage_of(plan, rank)
    acquired: dict[str, dict] = {}
    for route in plan.state_routes:
        if route.donor_kind == "checkpoint" or rollback:
            if rank in route.target_ranks:
                acquired.update(_anchor_slices(config, route, anchor, rank))
            continue
        acquired.update(_route_transfer(config, route, local, rank, group=groups.live, device=tdev))
    if stage is None:
        return None
    owned = stage_layout(plan, stage)
    idx = stage.tp_members.index(rank)
    state: dict[str, dict] = {}
    for name, dim in owned.items():
        if name in acquired:
            state[name] = acquired[name]
        elif rollback:
            e = anchor[name]
            state[name] = {f: local_slice(e[f], dim, idx, stage.tp_degree) for f in FIELDS if f in e}
            if "step" in e:
                state[name]["step"] = e["step"]
        elif name in local:
            state[name] = local[name]
        else:
            raise ReshardError(f"no state route covers {name} for rank {rank}")
    return PlannedRun(
        plan, rank=rank, local_state={n: f["param"] for n, f in state.items()},
        moments={n: f for n, f in state.items() if "exp_avg" in f}, groups=groups, device=device,
        cursor=completed if rollback else cursor, pin=pin,
    )


def _p2p_recover(run, *, plan, rank, anchor, groups, device, cursor, pin):
    """The CUDA path: new owners pull their shards from the donors' regions over NVLink.

    Every surviving rank publishes its flat-state region (IPC handle, field and tensor
    offsets, AdamW step) over the world group; each rank of the new plan builds its stage
    with an unfilled region and moves every owned tensor with one ``reshard_gather``
    launch: pieces of peer routes from the donors' regions (re-chunked for the new TP
    degree inside the copy descriptors), tensors it keeps from its own old region, and
    ``checkpoint`` routes from the host anchor. A barrier over the world group then tells
    the donors that nothing reads their regions any more.
    """
    from .ops import check_device_errors

    config = plan.config
    k = _ext.require()
    mine = None if run is None else run.stage.flat.export()
    gathered = [None] * dist.get_world_size(groups.world)
    dist.all_gather_object(gathered, (rank, mine), group=groups.world)
    regions = {r: m for r, m in gathered if m is not None}
    stage = stage_of(plan, rank)
    new_run = None
    opened: dict[int, int] = {}
    try:
        if stage is not None:
            new_run = PlannedRun(plan, rank=rank, local_state=None, moments=None, groups=groups, device=device,
                                 cursor=cursor, pin=pin)
            flat = new_run.stage.flat
            shapes = _shape_of(config)
            owned = stage_layout(plan, stage)
            by_name = {}
            for route in routes_for(plan, rank):
                for name in route_names(config, route):
                    by_name[name] = route

            def region_of(r):
                if r == rank:
                    if run is None:
                        raise ReshardError(f"rank {rank} is named as a donor but holds no state")
                    return run.stage.flat.region_ptr
                if r not in regions:
                    raise ReshardError(f"donor rank {r} published no state")
                if r not in opened:
                    opened[r] = k.symm_open(regions[r]["handle"])
                return opened[r]

            gp = peer.GatherPlan()
            host: dict[str, dict] = {}
            steps = set()
            for name, dim in owned.items():
                dst_off = flat.offsets[name][0]
                route = by_name.get(name)
                if route is not None and route.donor_kind == "checkpoint":
                    host[name] = _anchor_slices(config, route, anchor, rank)[name]
                    if "step" in host[name]:
                        steps.add(int(float(host[name]["step"])))
                    continue
                if route is not None:
                    pieces = peer.shard_pieces(shapes[name], dim, route.donor_degree, route.target_degree,
                                               route.target_ranks.index(rank))
                    donors = route.donor_ranks
                else:
                    if run is None or name not in run.stage.flat.offsets:
                        raise ReshardError(f"no state route covers {name} for rank {rank}")
                    n = run.stage.flat.offsets[name][1]
                    count = 1
                    for x in n:
                        count *= int(x)
                    pieces = [peer.Piece(0, 0, count, 0, count, 1, count)]
                    donors = (rank,)
                for piece in pieces:
                    donor = donors[piece.donor]
                    meta = regions.get(donor) if donor != rank else mine
                    if meta is None or name not in meta["offsets"]:
                        raise ReshardError(f"donor rank {donor} does not hold {name}")
                    gp.add([piece], src_region=region_of(donor), src_fields=meta["fields"],
                           src_tensor_off=meta["offsets"][name], dst_flat=flat, dst_tensor_off=dst_off)
                    steps.add(int(meta["step"]))
            gp.launch(flat.master.device)
            with torch.no_grad():
                for name, entry in host.items():
                    for f, buf in (("param", flat.master), ("exp_avg", flat.exp_avg), ("exp_avg_sq", flat.exp_avg_sq)):
                        if f in entry:
                            flat.view(buf, name).copy_(entry[f].to(buf.device))
                    if flat.work is not flat.master:
                        flat.view(flat.work, name).copy_(flat.view(flat.master, name))
            torch.cuda.synchronize(flat.master.device)
            check_device_errors(flat.master.device.index or 0)
            if len(steps) > 1:
                raise ReshardError(f"donors disagree on the AdamW step: {sorted(steps)}")
            flat.step = steps.pop() if steps else 0
    finally:
        # Everyone's gathers are done before any donor region may be released.
        dist.barrier(group=groups.world)
        for ptr in opened.values():
            k.symm_close(ptr)
    return new_run


def recover(run, *, plan, previous, rank, cursor, checkpoint_path, groups: TrainingGroups, device=None, pin=False):
    """Safe-point step 7: execute ``plan``'s state routes.

    Returns ``(run, state digest, resume cursor)``: the cursor is the number of completed
    iterations training continues from -- ``cursor`` itself, or the checkpoint's count
    when the plan needs a checkpoint route and the checkpoint is older than the live
    state (every rank then rolls back to it). A failure before the first commit of a
    ``checkpoint_every > 1`` run rolls back to the seeded initial state
    (:class:`InitialAnchor`, cursor 0); a missing file after a commit is
    ``checkpoint_unusable``.

    Every surviving rank calls this (the idle ones too: their shards may be donors).
    The checkpoint is read only when some route needs it or when it is current, in which
    case it is also the A1 oracle; otherwise the agreed digest covers every rank's shard
    fingerprint.
    """
    config = plan.config
    needs_checkpoint = any(r.donor_kind == "checkpoint" for r in plan.state_routes)
    loaded = _load_anchor(checkpoint_path)
    if loaded is None and needs_checkpoint:
        if cursor >= config.checkpoint_every:  # a commit happened, and its file is gone
            raise CheckpointError(f"checkpoint missing: {checkpoint_path}")
        # no commit yet (checkpoint_every > 1): the seeded initial state is the checkpoint
        initial = InitialAnchor(config, device)
        loaded = (initial, 0, initial.digest)
    anchor, completed, ck_digest = loaded if loaded is not None else ({}, None, None)
    current = completed == cursor
    rollback = needs_checkpoint and not current
    local = {} if run is None or rollback else run.local_state()
    tdev = torch.device("cpu") if device is None else torch.device(device)

    p2p = (tdev.type == "cuda" and config.dtype == "bf16" and peer.ENABLED and not rollback)
    if p2p:
        new_run = _p2p_recover(run, plan=plan, rank=rank, anchor=anchor, groups=groups, device=tdev,
                               cursor=cursor, pin=pin)
    else:
        new_run = _collective_recover(run, local, plan=plan, rank=rank, anchor=anchor, rollback=rollback,
                                      completed=completed, groups=groups, device=device, tdev=tdev, cursor=cursor,
                                      pin=pin)

    if current or rollback:
        if new_run is not None:
            problems = checkpoint_mismatches(new_run, plan=plan, rank=rank, anchor=anchor)
            if problems:
                raise ReshardError(f"rank {rank} state differs from the checkpoint: {problems[:5]}")
        return new_run, ck_digest, completed if rollback else cursor
    gathered = [None] * dist.get_world_size(groups.world)
    dist.all_gather_object(gathered, (rank, state_fingerprint(new_run)), group=groups.world)
    return new_run, sha256(repr(sorted(gathered)).encode("utf-8")).hexdigest(), cursor


def checkpoint_mismatches(run, *, plan, rank, anchor) -> list[str]:
    """Principle A1: every way this rank's state differs from the anchor's slices."""
    stage = stage_of(plan, rank)
    if stage is None:
        return [] if run is None else [f"rank {rank} is placed nowhere but still holds a run"]
    layout = stage_layout(plan, stage)
    shards = run.stage.local_shards()
    if set(shards) != set(layout):
        return [f"stage holds the wrong names: extra={sorted(set(shards) - set(layout))} "
                f"missing={sorted(set(layout) - set(shards))}"]
    idx = stage.tp_members.index(rank)
    problems = []
    for name, dim in layout.items():
        want = anchor[name]
        if not torch.equal(shards[name][0].detach().cpu(), local_slice(want["param"], dim, idx, stage.tp_degree)):
            problems.append(f"{name}.param")
        if "exp_avg" not in want:
            continue
        mv = run.stage.moment_views(name)
        for f in ("exp_avg", "exp_avg_sq"):
            if not torch.equal(mv[f].detach().cpu(), local_slice(want[f], dim, idx, stage.tp_degree)):
                problems.append(f"{name}.{f}")
        if float(run.stage.flat.step) != float(want["step"]):
            problems.append(f"{name}.step")
    return problems


def recovery_stop_code(error: Exception) -> str | None:
    if isinstance(error, CheckpointError):
        return "checkpoint_unusable"
    if isinstance(error, ReshardError):
        return "state_mismatch"
    return None


def run_from_anchor(plan, *, rank, anchor, completed, groups: TrainingGroups, device=None, pin=False):
    """A fresh run of ``plan`` whose state is the checkpoint ``anchor`` (cursor ``completed``).

    The uninterrupted re-run that a recovered run is compared against: the same plan, the
    same state, the same data cursor, started from scratch.
    """
    stage = stage_of(plan, rank)
    if stage is None:
        return None
    idx = stage.tp_members.index(rank)
    params, moments = {}, {}
    for name, dim in stage_layout(plan, stage).items():
        e = anchor[name]
        params[name] = local_slice(e["param"], dim, idx, stage.tp_degree)
        if "exp_avg" in e:
            moments[name] = {
                "exp_avg": local_slice(e["exp_avg"], dim, idx, stage.tp_degree),
                "exp_avg_sq": local_slice(e["exp_avg_sq"], dim, idx, stage.tp_degree),
                "step": e["step"],
            }
    return PlannedRun(plan, rank=rank, local_state=params, moments=moments, groups=groups, device=device,
                      cursor=completed, pin=pin)
