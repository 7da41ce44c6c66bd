"""Logical-state resharding by full-tensor reconstruction: the general, any-layout path.

Recovery itself moves state with the plan's routes (peer-to-peer gather kernels on the
GPU, one collective per route on the CPU path; :mod:`resihp.recovery`). This module
keeps the reference's functional interface (``resihp/parallel/reshard.py:36-243``) for
code that holds shards in hand and wants them at another TP degree:

* :func:`shard_dims` -- logical name -> TP shard dim, from the single layout table
  (:mod:`resihp.models.layout`);
* :func:`reconstruct_full` -- one full tensor from the shards on hand, else the
  checkpoint, else :class:`ReshardError`;
* :func:`local_slice` / :func:`shard_logical_state` -- cut a full state to one rank;
* :func:`reshard_tp_state` -- every rank of a group contributes the shards it holds
  (at whatever degree each was cut), every rank rebuilds the same full state, and each
  keeps its slice under the new degree; optionally checked against a checkpoint.

It exchanges whole shards as Python objects over ``group`` (Gloo or NCCL), so it suits
small states, tests and tools; it is not the recovery fast path.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..config import TrainConfig
from ..models import layout as _layout
from .tp import local_slice

#: Fields resharded like the parameter; ``step`` is a replicated scalar.
SHARDED_FIELDS = ("param", "exp_avg", "exp_avg_sq")
REPLICATED_FIELDS = ("step",)


class ReshardError(RuntimeError):
    """State could not be recovered intact (stop code ``state_mismatch``)."""


def shard_dims(layer_ids, config: TrainConfig | None = None) -> dict[str, int | None]:
    """Logical name -> shard dim (``None`` = replicated) for the given layers plus the
    embedding and head. Without ``config`` the names are the GPT-2 blocks'."""
    ids = list(layer_ids)
    if config is None:
        config = TrainConfig(model_dim=8, num_layers=max(ids, default=0) + 1, num_heads=1, batch_size=1,
                             micro_batch_size=1, seed=1, tp=1, pp=1, dp=1, iterations=1)
    return _layout.shard_dims(config, ids)


def reconstruct_full(name: str, shard_dim: int | None, old_size: int, contributions: dict, checkpoint=None):
    """``(full tensor, "peer" | "checkpoint")`` for one logical tensor.

    ``contributions`` maps shard index -> shard at degree ``old_size``. A replicated
    tensor needs any one copy (the lowest index is taken); a sharded one needs all
    ``old_size`` indices, concatenated along ``shard_dim``. Otherwise ``checkpoint[name]``
    is used when present; failing both, the tensor is lost: :class:`ReshardError`.
    """
    if shard_dim is None and contributions:
        return contributions[min(contributions)], "peer"
    if shard_dim is not None and old_size > 0 and all(i in contributions for i in range(old_size)):
        return torch.cat([contributions[i] for i in range(old_size)], dim=shard_dim), "peer"
    if checkpoint is not None and name in checkpoint:
        return checkpoint[name], "checkpoint"
    raise ReshardError(f"logical tensor {name} unavailable from peers and checkpoint")


def shard_logical_state(full_state: dict, *, layout: dict, tp_rank: int, tp_size: int) -> dict:
    """``{name: full tensor}`` cut to rank ``tp_rank`` of ``tp_size`` for every name of ``layout``."""
    return {name: local_slice(full_state[name], dim, tp_rank, tp_size) for name, dim in layout.items()}


def _portable(local_state: dict, default_count: int) -> dict:
    """``{name: {field: (index, count, cpu tensor)}}`` -- what one rank contributes."""
    out = {}
    for name, entry in local_state.items():
        index = int(entry.get("shard_index", 0))
        count = int(entry.get("shard_count", default_count))
        fields = {}
        for f in SHARDED_FIELDS + REPLICATED_FIELDS:
            if f in entry:
                v = entry[f]
                v = v.detach().to("cpu") if torch.is_tensor(v) else torch.tensor(float(v))
                fields[f] = (index, count, v)
        out[name] = fields
    return out


def _pool(contributions: list) -> dict:
    """name -> field -> shard count -> {index: tensor}, over every rank's contribution."""
    pool: dict = {}
    for contribution in contributions:
        for name, fields in contribution.items():
            for f, (index, count, tensor) in fields.items():
                pool.setdefault(name, {}).setdefault(f, {}).setdefault(count, {}).setdefault(index, tensor)
    return pool


def _rebuild(name: str, dim, old_size: int, by_count: dict, fallback):
    """Prefer shards cut at ``old_size``, then any other complete degree (ascending),
    then the checkpoint."""
    order = ([old_size] if old_size in by_count else []) + sorted(c for c in by_count if c != old_size)
    for count in order:
        shards = by_count[count]
        if dim is None or all(i in shards for i in range(count)):
            return reconstruct_full(name, dim, count, shards)
    return reconstruct_full(name, dim, old_size, {}, None if fallback is None else {name: fallback})


def reshard_tp_state(local_state: dict, *, layout: dict, old_size: int, new_size: int, new_rank: int | None,
                     group=None, checkpoint: dict | None = None, verify: bool = True) -> dict:
    """Re-cut param and AdamW state to a new TP degree / membership.

    ``local_state``: ``{name: {"shard_index", ["shard_count"], "param", "exp_avg",
    "exp_avg_sq", "step"}}`` for the shards this rank holds (``{}`` if none); a missing
    ``shard_count`` means ``old_size``. Every rank of ``group`` calls this and rebuilds
    the same full state; ``new_rank`` is this rank's index in the new TP group of size
    ``new_size``, or ``None`` for a rank that only donates. ``checkpoint``
    (``{name: {field: full tensor}}``) fills tensors no peer holds and, with ``verify``,
    must equal every peer reconstruction (:class:`ReshardError` otherwise). Returns
    ``{name: {field: new shard}}`` (empty for a donating-only rank).
    """
    world = dist.get_world_size(group)
    gathered: list = [None] * world
    dist.all_gather_object(gathered, _portable(local_state, old_size), group=group)
    pool = _pool(gathered)

    out: dict = {}
    for name, dim in layout.items():
        saved = None if checkpoint is None else checkpoint.get(name)
        rebuilt = {}
        for f in SHARDED_FIELDS + REPLICATED_FIELDS:
            by_count = pool.get(name, {}).get(f, {})
            fallback = None if saved is None else saved.get(f)
            if not by_count and fallback is None:
                continue
            fdim = None if f in REPLICATED_FIELDS else dim
            full, source = _rebuild(name, fdim, old_size, by_count, fallback)
            if verify and source == "peer" and fallback is not None and not torch.equal(full, fallback):
                raise ReshardError(f"reshard verify failed for {name}.{f}")
            rebuilt[f] = full
        if new_rank is not None:
            out[name] = {f: local_slice(t, None if f in REPLICATED_FIELDS else dim, new_rank, new_size)
                         for f, t in rebuilt.items()}
    return out
