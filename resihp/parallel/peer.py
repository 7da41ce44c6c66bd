"""Peer access to the flat training-state regions (CUDA IPC over NVLink).

On the CUDA kernel path every stage keeps its flat state in one IPC-exported region
(:class:`~resihp.parallel.tp.FlatState` with ``shared=True``). Two consumers map the
regions of other ranks and read them with P2P loads inside their own kernels:

* :class:`DpPeers` -- the fused data-parallel step: gradient all-reduce over the DP
  position group, AdamW and the bf16 refresh in one launch (``dp_allreduce_adamw``).
  It replaces the reference's CPU object gather of full gradients
  (``resihp/parallel/dp.py:98-151``) followed by ``optimizer.step()``
  (``resihp/parallel/pp.py:428-451``).
* :func:`shard_pieces` / :class:`GatherPlan` -- the post-failure state move: each new
  owner pulls the pieces of its new shards straight from the donors' regions, the
  re-partition (shard dim 0 or 1, any old and new TP degree) expressed as strided copy
  descriptors, one ``reshard_gather`` launch per rank (reference: the all-gather-object
  reshard of ``resihp/parallel/reshard.py:187-243``).
* :class:`HeteroPeers` -- the logical gradient sum for replicas with different layouts
  (reference: ``resihp/parallel/dp.py:140-151``) as P2P pulls of the other holders'
  pieces plus an ordered sum (``RESIHP_P2P_HETERO=0``: bucketed NCCL all-reduces instead).

Mappings are opened after a fail-stop's world re-formation and closed at the next safe
point, when no kernel is in flight; a dead rank's region is never mapped again.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..ops import _ext

ENABLED = os.environ.get("RESIHP_FUSED_DP", "1") != "0"
# Groups of at least this many replicas take the two-phase kernel (each rank reduces one
# part of every slice and pushes the sum to all ranks): 2 (dp-1)/dp of the gradient
# bytes cross NVLink into each GPU instead of (dp-1) times them.
PUSH_MIN_DP = int(os.environ.get("RESIHP_DP_PUSH_MIN", "3"))
MAX_DP = 8
DP_FLAG_OFFSET = 0          # byte offset of the DP flag words inside the region's flag area
COPY_ROW = 32 * 1024        # longest row (elements) one copy work item moves


# ---------------------------------------------------------------------------------------
# data parallelism
# ---------------------------------------------------------------------------------------


class DpPeers:
    """This rank's mappings of its DP peers' regions and the fused step over them.

    Every rank of ``group`` holds a byte-identical flat layout (homogeneous replicas), so
    element ``i`` of every region is the same logical value. Group ranks are ordered by
    global rank, which fixes the summation order of the reduction on every replica.
    """

    def __init__(self, stage, group):
        k = _ext.require()
        flat = stage.flat
        if not flat.shared:
            raise ValueError("the fused DP step needs the shared flat-state region")
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.size > MAX_DP:
            raise ValueError(f"fused DP step supports up to {MAX_DP} replicas")
        meta = flat.export()
        gathered = [None] * self.size
        dist.all_gather_object(gathered, meta, group=group)
        for other in gathered:
            if other["numel"] != flat.numel or other["fields"] != meta["fields"] or other["offsets"] != meta["offsets"]:
                raise ValueError("DP peers hold different flat layouts")
        self.device = flat.master.device
        self.bases = []
        with torch.cuda.device(self.device):
            for r, other in enumerate(gathered):
                self.bases.append(flat.region_ptr if r == self.rank else k.symm_open(other["handle"]))
        self.grid = k.dp_grid(flat.numel, self.device.index or 0)
        self.push = self.size >= PUSH_MIN_DP
        if DP_FLAG_OFFSET + 2 * 4 * MAX_DP * self.grid > flat.flags.numel() * 4:
            raise ValueError("DP flag area too small for the launch grid")
        self.epoch = 0
        self.closed = False

    def step(self, stage) -> None:
        """Sum the accumulated gradients over the group and take the AdamW step."""
        k = _ext.require()
        flat = stage.flat
        c = stage.config
        self.epoch += 1
        flat.step += 1
        cur = flat.parity
        goff = flat.field_offsets[f"grad{cur}"]
        foff = DP_FLAG_OFFSET  # the flag area starts the region
        extra = {}
        if self.push:
            soff = flat.field_offsets[f"grad{1 - cur}"]
            f2 = foff + 4 * MAX_DP * self.grid  # the second flag array follows the first
            extra = dict(sums_peer=[b + soff for b in self.bases], flags2_local=flat.region_ptr + f2,
                         flags2_peer=[b + f2 for b in self.bases])
        k.dp_allreduce_adamw(
            [b + goff for b in self.bases], self.rank, flat.grads[1 - cur], flat.master, flat.exp_avg,
            flat.exp_avg_sq, None if flat.work is flat.master else flat.work, c.lr, c.beta1, c.beta2, c.adam_eps,
            c.weight_decay, flat.step, 1.0, flat.region_ptr + foff, [b + foff for b in self.bases], self.epoch,
            self.grid, **extra,
        )
        stage.use_grad(1 - cur)

    def close(self, *, barrier: bool = True) -> None:
        """Unmap the peers' regions (every rank's kernels must be done: see ``barrier``)."""
        if self.closed:
            return
        k = _ext.require()
        torch.cuda.synchronize(self.device)
        if barrier:
            dist.barrier(group=self.group)
        for r, base in enumerate(self.bases):
            if r != self.rank:
                k.symm_close(base)
        self.closed = True


# ---------------------------------------------------------------------------------------
# the state move (pure piece arithmetic + one gather launch)
# ---------------------------------------------------------------------------------------


def chunk_bounds(length: int, parts: int, index: int) -> tuple[int, int]:
    """``torch.chunk``'s split of ``length`` into ``parts``: the range of piece ``index``."""
    size = -(-length // parts)
    return min(index * size, length), min((index + 1) * size, length)


@dataclass(frozen=True)
class Piece:
    """One strided block of a target shard and where it comes from (element units).

    Rows ``r < rows`` copy ``cols`` elements from ``src_off + r * src_ld`` of donor
    ``donor``'s shard to ``dst_off + r * dst_ld`` of the target shard.
    """

    donor: int
    src_off: int
    src_ld: int
    dst_off: int
    dst_ld: int
    rows: int
    cols: int


def _numel(shape) -> int:
    n = 1
    for x in shape:
        n *= int(x)
    return n


def shard_pieces(shape, dim, donor_degree: int, target_degree: int, target_index: int) -> list[Piece]:
    """The blocks of target shard ``target_index`` (of ``target_degree``) cut from the
    ``donor_degree`` donor shards of a tensor of logical ``shape`` split along ``dim``.

    ``dim=None`` (replicated): the whole tensor from donor 0. Pieces follow
    ``torch.chunk`` boundaries on both sides, so any pair of degrees works.
    """
    if dim is None:
        n = _numel(shape)
        return [Piece(0, 0, n, 0, n, 1, n)]
    outer = _numel(shape[:dim])
    length = int(shape[dim])
    inner = _numel(shape[dim + 1:])
    ta, tb = chunk_bounds(length, target_degree, target_index)
    out = []
    for i in range(donor_degree):
        da, db = chunk_bounds(length, donor_degree, i)
        a, b = max(ta, da), min(tb, db)
        if a >= b:
            continue
        src_ld, dst_ld, cols = (db - da) * inner, (tb - ta) * inner, (b - a) * inner
        src_off, dst_off = (a - da) * inner, (a - ta) * inner
        if outer == 1 or (src_ld == cols and dst_ld == cols):
            out.append(Piece(i, src_off, outer * cols, dst_off, outer * cols, 1, outer * cols))
        else:
            out.append(Piece(i, src_off, src_ld, dst_off, dst_ld, outer, cols))
    return out


def split_rows(piece: Piece, limit: int = COPY_ROW) -> list[Piece]:
    """Cut a single long contiguous row into rows of at most ``limit`` elements."""
    if piece.rows != 1 or piece.cols <= limit:
        return [piece]
    full, rest = divmod(piece.cols, limit)
    out = [Piece(piece.donor, piece.src_off, limit, piece.dst_off, limit, full, limit)]
    if rest:
        tail = full * limit
        out.append(Piece(piece.donor, piece.src_off + tail, rest, piece.dst_off + tail, rest, 1, rest))
    return out


def apply_pieces(pieces, donors: list[torch.Tensor], target: torch.Tensor) -> None:
    """Host/any-device execution of ``pieces`` with torch ops (the CPU path and the oracle)."""
    flat_t = target.reshape(-1)
    for p in pieces:
        src = donors[p.donor].reshape(-1)
        for r in range(p.rows):
            s0, d0 = p.src_off + r * p.src_ld, p.dst_off + r * p.dst_ld
            flat_t[d0: d0 + p.cols].copy_(src[s0: s0 + p.cols])


class GatherPlan:
    """Copy descriptors of one rank's state move, executed by one ``reshard_gather``."""

    FIELDS = ("master", "exp_avg", "exp_avg_sq")

    def __init__(self):
        self.rows: list[list[int]] = []
        self.items = 0

    def add(self, pieces, *, src_region: int, src_fields: dict, src_tensor_off: int, dst_flat, dst_tensor_off: int):
        """Queue ``pieces`` of one logical tensor for all three state fields.

        ``src_region`` is the (mapped or own) base address of the donor's region,
        ``src_fields``/``src_tensor_off`` its field offsets (bytes) and the tensor's
        element offset in the donor's flat layout; ``dst_flat`` is the new FlatState.
        """
        dst_base = dst_flat.region_ptr
        for piece in pieces:
            for p in split_rows(piece):
                for f in self.FIELDS:
                    src = src_region + src_fields[f] + 4 * (src_tensor_off + p.src_off)
                    dst = dst_base + dst_flat.field_offsets[f] + 4 * (dst_tensor_off + p.dst_off)
                    bf16 = 0
                    if f == "master" and dst_flat.work is not dst_flat.master:
                        bf16 = dst_base + dst_flat.field_offsets["work"] + 2 * (dst_tensor_off + p.dst_off)
                    vec4 = int(src % 16 == 0 and dst % 16 == 0 and p.src_ld % 4 == 0 and p.dst_ld % 4 == 0
                               and p.cols % 4 == 0 and (bf16 % 8 == 0))
                    self.rows.append([src, dst, bf16, p.src_ld, p.dst_ld, p.rows, p.cols, self.items, vec4])
                    self.items += p.rows

    def add_field(self, pieces, *, src_base: int, dst_base: int) -> None:
        """Queue ``pieces`` of one FP32 field: ``src_base`` / ``dst_base`` are the byte
        addresses of element 0 of the donor's and of the target's tensor."""
        for piece in pieces:
            for p in split_rows(piece):
                src = src_base + 4 * p.src_off
                dst = dst_base + 4 * p.dst_off
                vec4 = int(src % 16 == 0 and dst % 16 == 0 and p.src_ld % 4 == 0 and p.dst_ld % 4 == 0
                           and p.cols % 4 == 0)
                self.rows.append([src, dst, 0, p.src_ld, p.dst_ld, p.rows, p.cols, self.items, vec4])
                self.items += p.rows

    def launch(self, device) -> None:
        if not self.rows:
            return
        table = torch.tensor(self.rows, dtype=torch.int64).to(device)
        _ext.require().reshard_gather(table, self.items)
        self._keep = table  # alive until the launch has run (the caller synchronises)


# ---------------------------------------------------------------------------------------
# heterogeneous replicas: the logical gradient sum by P2P pulls
# ---------------------------------------------------------------------------------------

HETERO_ENABLED = os.environ.get("RESIHP_P2P_HETERO", "1") == "1"


@dataclass(frozen=True)
class StageMeta:
    """What every executor publishes about its stage for the heterogeneous reduction."""

    rank: int
    replica: int
    stage: int
    tp_members: tuple[int, ...]
    layout: dict          # {name: shard dim or None}
    export: dict          # FlatState.export(): handle, field offsets, tensor offsets


def hetero_terms(metas: dict, rank: int, shapes: dict) -> list[tuple[str, int, list]]:
    """For each tensor ``rank`` owns: ``(name, own position, [(position, donor rank, Piece)])``.

    The logical gradient of a tensor is the sum over every *holder stage* (each replica's
    stage that holds it, twice per replica for tied embeddings) of that stage's full
    gradient. Holders are ordered by (replica, stage); a rank's shard of the sum is the
    same positions of every holder's contribution, cut from the holder's TP shards by
    :func:`shard_pieces` (a replicated tensor from the holder's first TP rank).
    """
    me = metas[rank]
    stages = {}
    for m in metas.values():
        stages.setdefault((m.replica, m.stage), m)
    ordered = [stages[k] for k in sorted(stages)]
    my_index = me.tp_members.index(rank)
    out = []
    for name, dim in sorted(me.layout.items()):
        holders = [s for s in ordered if name in s.layout]
        own = next(i for i, s in enumerate(holders) if (s.replica, s.stage) == (me.replica, me.stage))
        terms = []
        for pos, h in enumerate(holders):
            if pos == own:
                continue
            for piece in shard_pieces(shapes[name], dim, len(h.tp_members), len(me.tp_members), my_index):
                terms.append((pos, h.tp_members[piece.donor], piece))
        out.append((name, own, terms))
    return out


def hetero_gather(terms, metas: dict, rank: int, flat, region_of, scratch) -> tuple[GatherPlan, list[dict]]:
    """Copy descriptors pulling every other holder's pieces of this rank's shards into
    ``scratch`` rows (one row per holder position, laid out like this rank's flat state);
    ``region_of(rank)`` is the address of a rank's region here. Returns the descriptors
    and, per term list, ``{holder position: scratch row}``."""
    plan = GatherPlan()
    slots = []
    for name, _own, pieces in terms:
        slot = {p: i for i, p in enumerate(sorted({p for p, _d, _q in pieces}))}
        slots.append(slot)
        dst_off = flat.offsets[name][0]
        for pos, donor, piece in pieces:
            m = metas[donor]
            src = region_of(donor) + m.export["fields"]["grad0"] + 4 * m.export["offsets"][name]
            plan.add_field([piece], src_base=src, dst_base=scratch[slot[pos]].data_ptr() + 4 * dst_off)
    return plan, slots


def hetero_sum(terms, slots, scratch, flat, grad) -> None:
    """Overwrite each shard in ``grad`` (this rank's gradient buffer) with the sum of the
    holders' contributions, added in holder order."""
    with torch.no_grad():
        for (name, own, pieces), slot in zip(terms, slots):
            if not pieces:
                continue
            g = flat.view(grad, name)
            off, shape = flat.offsets[name]
            parts = [g if pos == own else scratch[slot[pos]][off: off + g.numel()].view(shape)
                     for pos in range(len(slot) + 1)]
            acc = parts[0].clone()
            for t in parts[1:]:
                acc.add_(t)
            g.copy_(acc)


class HeteroPeers:
    """P2P logical gradient sum for replicas with different layouts (after fail-stops).

    Each executor maps every other executor's flat-state region. Per step: every rank
    synchronises and meets the others at a barrier (all gradients final), pulls the
    pieces of the other holders' gradients of its own shards into a scratch buffer with
    one gather launch, meets them again (all pulls done), and sums the holders'
    contributions in (replica, stage) order into its gradient -- the same order on every
    rank that holds an element, so the sums agree bit for bit. Replaces the per-tensor
    full-size all-reduce of the collective path.
    """

    def __init__(self, stage, plan, rank, group):
        from ..models.layout import model_specs
        from ..recovery import stage_layout, stage_of

        k = _ext.require()
        flat = stage.flat
        if not flat.shared:
            raise ValueError("the P2P heterogeneous reduction needs the shared flat-state region")
        sp = stage_of(plan, rank)
        mine = StageMeta(rank, sp.replica_id, sp.stage_id, tuple(sp.tp_members), stage_layout(plan, sp), flat.export())
        gathered = [None] * dist.get_world_size(group)
        dist.all_gather_object(gathered, mine, group=group)
        metas = {m.rank: m for m in gathered}
        self.group = group
        self.rank = rank
        self.device = flat.master.device
        shapes = {s.name: s.shape for s in model_specs(plan.config)}
        self.terms = hetero_terms(metas, rank, shapes)
        slots = max((len({p for p, _d, _q in t}) for _n, _o, t in self.terms), default=0)
        self.scratch = torch.zeros((max(slots, 1), flat.numel), dtype=torch.float32, device=self.device)
        self.opened = {}
        with torch.cuda.device(self.device):
            for r, m in metas.items():
                if r != rank:
                    self.opened[r] = k.symm_open(m.export["handle"])
        self.plan, self.slot_of = hetero_gather(
            self.terms, metas, rank, flat, lambda r: flat.region_ptr if r == rank else self.opened[r], self.scratch)
        self.table = None
        self.closed = False

    def reduce(self, stage) -> None:
        if stage.flat.parity != 0:
            raise RuntimeError("the heterogeneous reduction reads gradient buffer 0")
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)              # every holder's gradients are final
        if self.plan.rows:
            if self.table is None:
                self.table = torch.tensor(self.plan.rows, dtype=torch.int64).to(self.device)
            _ext.require().reshard_gather(self.table, self.plan.items)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)              # nobody reads a gradient any more
        hetero_sum(self.terms, self.slot_of, self.scratch, stage.flat, stage.flat.grads[0])

    def close(self, *, barrier: bool = True) -> None:
        if self.closed:
            return
        k = _ext.require()
        torch.cuda.synchronize(self.device)
        if barrier:
            dist.barrier(group=self.group)
        for ptr in self.opened.values():
            k.symm_close(ptr)
        self.closed = True
