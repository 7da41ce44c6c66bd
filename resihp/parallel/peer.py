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
        if DP_FLAG_OFFSET + 4 * MAX_DP * self.grid > flat.flags.numel() * 4:
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
        k.dp_allreduce_adamw(
            [b + goff for b in self.bases], self.rank, flat.grads[1 - cur], flat.master, flat.exp_avg,
            flat.exp_avg_sq, None if flat.work is flat.master else flat.work, c.lr, c.beta1, c.beta2, c.adam_eps,
            c.weight_decay, flat.step, 1.0, flat.region_ptr + foff, [b + foff for b in self.bases], self.epoch,
            self.grid,
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

    def launch(self, device) -> None:
        if not self.rows:
            return
        table = torch.tensor(self.rows, dtype=torch.int64).to(device)
        _ext.require().reshard_gather(table, self.items)
        self._keep = table  # alive until the launch has run (the caller synchronises)
