"""Data-parallel routing and the cross-holder gradient reduction.

Routing (reference ``resihp/parallel/dp.py:32-95``): every ``(micro_batch, stage)``
names its executors in the plan's :class:`~resihp.planner.dp.DPAssignment`;
:func:`executor_route` turns that into this rank's micro-batches and the actual
upstream / downstream executors, which may sit in another replica after a reroute.

Gradient reduction. Semantics are the reference's ``dp_combine_gradients`` (sum every
logical gradient over every copy that holds it, whatever TP degree or PP layout each
replica runs), extended to tied embeddings (the embedding stage and the head stage of
one replica are two holders of ``token_embedding.weight``). Two executions:

* **homogeneous plans** (every replica has the same stage ranges and TP degrees; the
  common case and the benchmark): the flat gradient buffers of the ``(stage, TP rank)``
  positions are byte-compatible across replicas, so one all-reduce per position group
  sums them; tied copies are summed first within each replica. Under sequence
  parallelism the replicated (norm) weights' gradients are partial sums over token
  shards and are all-reduced over the TP group first.
* **heterogeneous plans** (after a fail-stop left replicas at different degrees or
  layerings): each logical tensor is assembled at full size on every executor --
  every TP shard of every holder placed at its slice, a replicated tensor contributed
  once per holder -- and summed with one all-reduce over the executor group, then each
  rank keeps its own slice. The reference does the same with a CPU object gather.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..models.layout import model_specs


def stage_pipeline(assignment, micro_batch):
    placements = assignment.by_micro_batch[micro_batch]
    return tuple(sorted(placements, key=lambda p: p.stage_id))


def executor_route(assignment, rank):
    """Per micro-batch this rank executes: its stage's executors and its neighbours."""
    out = []
    for mb in sorted(assignment.by_micro_batch):
        chain = stage_pipeline(assignment, mb)
        for i, p in enumerate(chain):
            if rank not in p.executor_ranks:
                continue
            out.append(
                {
                    "micro_batch": mb,
                    "stage_id": p.stage_id,
                    "executors": p.executor_ranks,
                    "upstream": chain[i - 1].executor_ranks if i > 0 else None,
                    "downstream": chain[i + 1].executor_ranks if i < len(chain) - 1 else None,
                }
            )
    return out


def global_micro_count(assignment) -> int:
    return len(assignment.by_micro_batch)


class ActivationLog:
    """Activations retained from their forward until the matching backward."""

    def __init__(self):
        self.live: set = set()
        self.peak = 0

    def retain(self, key):
        self.live.add(key)
        self.peak = max(self.peak, len(self.live))

    def release(self, key):
        if key not in self.live:
            raise KeyError(f"release of activation {key} that is not live")
        self.live.discard(key)


# ---------------------------------------------------------------------------------------
# reduction topology (pure: derived from the plan, shared by the control plane)
# ---------------------------------------------------------------------------------------


@dataclass(frozen=True)
class ReductionTopology:
    homogeneous: bool
    dp_groups: tuple[tuple[int, ...], ...]      # same (stage, tp index) across replicas
    tied_groups: tuple[tuple[int, ...], ...]    # (embedding-stage rank, head-stage rank) per replica/tp index


def _replica_layouts(plan):
    out: dict[int, list] = {}
    for s in plan.stages:
        out.setdefault(s.replica_id, []).append(s)
    return {r: sorted(v, key=lambda s: s.stage_id) for r, v in out.items()}


def reduction_topology(plan) -> ReductionTopology:
    """Which groups the fast gradient reduction needs under ``plan`` (pure)."""
    layouts = _replica_layouts(plan)
    shapes = {r: tuple((s.stage_id, s.tp_degree, s.layer_range) for s in v) for r, v in layouts.items()}
    homogeneous = len(set(shapes.values())) == 1
    tied_ok = True
    if plan.config.tied_embeddings:
        for v in layouts.values():
            if len(v) > 1 and v[0].tp_degree != v[-1].tp_degree:
                tied_ok = False
    if not (homogeneous and tied_ok):
        return ReductionTopology(False, (), ())
    replicas = sorted(layouts)
    dp_groups = []
    first = layouts[replicas[0]]
    if len(replicas) > 1:
        for pos, stage in enumerate(first):
            for t in range(stage.tp_degree):
                dp_groups.append(tuple(sorted(layouts[r][pos].tp_members[t] for r in replicas)))
    tied = []
    if plan.config.tied_embeddings and len(first) > 1:
        for r in replicas:
            a, b = layouts[r][0], layouts[r][-1]
            for t in range(a.tp_degree):
                tied.append(tuple(sorted((a.tp_members[t], b.tp_members[t]))))
    return ReductionTopology(True, tuple(dp_groups), tuple(tied))


# ---------------------------------------------------------------------------------------
def dp_combine_gradients(local: dict, *, group=None) -> dict:
    """Sum each logical gradient over every replica that holds it; return this rank's
    slices of the sums (reference: ``resihp/parallel/dp.py:98-151``).

    ``local``: ``{name: {"grad", "shard_dim", "shard_index", "old_size", "replica"}}``
    for the shards this rank owns. Every rank of ``group`` exchanges its shards as
    objects; per name each replica's full gradient is rebuilt at that replica's own
    degree, the replicas are added in ascending replica id (so every rank adds the same
    terms in the same order), and each rank keeps its slice under its own layout. The
    general form for small states and tools; training reduces with
    :class:`GradientReducer`.
    """
    from .reshard import reconstruct_full
    from .tp import local_slice

    mine = {
        name: {"grad": e["grad"].detach().to("cpu"), "shard_dim": e["shard_dim"], "shard_index": int(e["shard_index"]),
               "old_size": int(e["old_size"]), "replica": int(e["replica"])}
        for name, e in local.items()
    }
    gathered: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(gathered, mine, group=group)
    shards: dict = {}  # name -> replica -> (degree, {index: grad})
    dims: dict = {}
    for contribution in gathered:
        for name, e in contribution.items():
            dims[name] = e["shard_dim"]
            degree, held = shards.setdefault(name, {}).setdefault(e["replica"], (e["old_size"], {}))
            held.setdefault(e["shard_index"], e["grad"])
    out = {}
    for name, e in local.items():
        total = None
        for replica in sorted(shards[name]):
            degree, held = shards[name][replica]
            full, _ = reconstruct_full(name, dims[name], degree, held)
            total = full.clone() if total is None else total + full
        out[name] = local_slice(total, e["shard_dim"], int(e["shard_index"]), int(e["old_size"])).to(e["grad"].device)
    return out


# the reducer
# ---------------------------------------------------------------------------------------


class GradientReducer:
    """Sums this rank's gradients with every other holder of the same logical tensors.

    ``groups`` maps each rank tuple of :func:`reduction_topology` to its process group
    (only the groups this rank belongs to); ``executor_group`` spans every active rank.
    """

    def __init__(self, plan, rank: int, *, groups: dict, executor_group=None, replica_id: int = 0):
        self.plan = plan
        self.rank = rank
        self.topology = reduction_topology(plan)
        self.groups = groups
        self.executor_group = executor_group
        self.replica_id = replica_id
        self.bucket_elems = 64 * 1024 * 1024
        self.fused_dp = None
        self.hetero = None

    def attach(self, stage) -> None:
        """Set up the fused DP step (one NVLink kernel: all-reduce + AdamW) where it applies.

        Collective over this rank's DP position group. Applies on the CUDA kernel path of
        a homogeneous plan; every rank decides the same way (config, device kind and the
        ``RESIHP_FUSED_DP`` switch are common to the job).
        """
        from . import peer

        if (not self.topology.homogeneous and peer.HETERO_ENABLED and stage.kernel and stage.flat.shared
                and self.executor_group is not None):
            stage.hetero = peer.HeteroPeers(stage, self.plan, self.rank, self.executor_group)
            self.hetero = stage.hetero
            return
        if not (peer.ENABLED and stage.kernel and stage.flat.shared and self.topology.homogeneous):
            return
        for members in self.topology.dp_groups:
            if self.rank in members and 1 < len(members) <= peer.MAX_DP:
                stage.dp = peer.DpPeers(stage, self.groups[members])
                self.fused_dp = stage.dp

    def reduce_and_step(self, stage) -> bool:
        """Reduce; with the fused DP step also take the optimizer step. True if stepped."""
        if self.fused_dp is None or self.fused_dp.closed:
            self.reduce(stage)
            return False
        self._sp_partial_replicated(stage)
        self._reduce_tied(stage)
        self.fused_dp.step(stage)
        return True

    def reduce(self, stage) -> None:
        if self.topology.homogeneous:
            self._reduce_fast(stage)
        elif self.hetero is not None and not self.hetero.closed:
            self._sp_partial_replicated(stage)
            self.hetero.reduce(stage)
        else:
            self._reduce_logical(stage)

    def _sp_partial_replicated(self, stage) -> None:
        if not stage.sp:
            return
        names = [s.name for s in stage.specs if s.shard_dim is None]
        if not names:
            return
        views = [stage.g[n] for n in names]
        buf = torch.cat([v.reshape(-1) for v in views])
        dist.all_reduce(buf, group=stage.group)
        off = 0
        for v in views:
            v.copy_(buf[off: off + v.numel()].view_as(v))
            off += v.numel()

    def _reduce_tied(self, stage) -> None:
        for members in self.topology.tied_groups:
            if self.rank in members:
                dist.all_reduce(stage.g["token_embedding.weight"], group=self.groups[members])

    def _reduce_fast(self, stage) -> None:
        self._sp_partial_replicated(stage)
        self._reduce_tied(stage)
        for members in self.topology.dp_groups:
            if self.rank in members:
                grad = stage.flat.grad
                for start in range(0, grad.numel(), self.bucket_elems):
                    dist.all_reduce(grad[start: start + self.bucket_elems], group=self.groups[members])

    def _reduce_logical(self, stage) -> None:
        """Heterogeneous plans: full-size logical sums over the executor group.

        Logical tensors are packed into buckets of about ``bucket_elems`` elements (one
        all-reduce per bucket, not per tensor); each tensor occupies the same bucket
        slot on every rank because the packing follows the model's name order.
        """
        if stage is not None:
            self._sp_partial_replicated(stage)
        config = self.plan.config
        device = stage.device if stage is not None else torch.device("cpu")
        held = {} if stage is None else {s.name: s for s in stage.specs}
        specs = model_specs(config)
        buckets, cur, size = [], [], 0
        for spec in specs:
            n = 1
            for x in spec.shape:
                n *= x
            cur.append((spec, n))
            size += n
            if size >= self.bucket_elems:
                buckets.append(cur)
                cur, size = [], 0
        if cur:
            buckets.append(cur)
        for bucket in buckets:
            flat = torch.zeros(sum(n for _s, n in bucket), dtype=torch.float32, device=device)
            off = 0
            for spec, n in bucket:
                full = flat[off: off + n].view(spec.shape)
                if spec.name in held:
                    if spec.shard_dim is None:
                        # one copy per holder stage: without SP every TP member computed the
                        # same gradient, with SP the partial sums were just all-reduced over
                        # the TP group, so either way each member holds the stage's total
                        if stage.tp_rank == 0:
                            full += stage.g[spec.name]
                    else:
                        torch.chunk(full, stage.tp_size, dim=spec.shard_dim)[stage.tp_rank].copy_(stage.g[spec.name])
                off += n
            dist.all_reduce(flat, group=self.executor_group)
            off = 0
            for spec, n in bucket:
                if spec.name in held:
                    full = flat[off: off + n].view(spec.shape)
                    mine = full if spec.shard_dim is None else torch.chunk(full, stage.tp_size, dim=spec.shard_dim)[stage.tp_rank]
                    stage.g[spec.name].copy_(mine)
                off += n
