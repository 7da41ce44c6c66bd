"""Piece arithmetic of the P2P state move (resihp.parallel.peer), checked on CPU.

For every (shape, shard dim, old degree, new degree, target index), executing the pieces
over the donor shards must reproduce exactly the target shard that ``local_slice`` cuts
from the full tensor -- the same contract the reference's reshard checks with
``torch.equal`` (``resihp/parallel/reshard.py:231-233``).
"""

import itertools

import pytest
import torch

from resihp.parallel.peer import Piece, apply_pieces, chunk_bounds, shard_pieces, split_rows
from resihp.parallel.tp import local_slice

SHAPES = [((48, 40), 0), ((48, 40), 1), ((40,), 0), ((40,), None), ((6, 8, 12), 1), ((6, 8, 12), 2), ((36, 20), None)]


def test_chunk_bounds_match_torch_chunk():
    for length, parts in itertools.product(range(1, 30), range(1, 9)):
        pieces = torch.chunk(torch.arange(length), parts)
        for i in range(parts):
            a, b = chunk_bounds(length, parts, i)
            want = pieces[i] if i < len(pieces) else torch.arange(0)
            assert torch.equal(torch.arange(a, b), want)


@pytest.mark.parametrize("shape,dim", SHAPES)
def test_pieces_rebuild_every_target_shard(shape, dim):
    full = torch.randn(shape)
    for old, new in itertools.product((1, 2, 4, 8), (1, 2, 4, 8)):
        if dim is not None and (shape[dim] % old or shape[dim] % new):
            continue
        donors = [local_slice(full, dim, i, old) for i in range(old)]
        for t in range(new):
            want = local_slice(full, dim, t, new)
            got = torch.full_like(want, float("nan"))
            pieces = shard_pieces(shape, dim, old, new, t)
            apply_pieces([q for p in pieces for q in split_rows(p, limit=7)], donors, got)
            assert torch.equal(got, want), (shape, dim, old, new, t)


def test_contiguous_pieces_are_single_runs():
    # dim 0 of a row-major tensor: every piece is one contiguous run
    for p in shard_pieces((64, 32), 0, 2, 4, 1):
        assert p.rows == 1
    # dim 1: strided rows
    pieces = shard_pieces((64, 32), 1, 4, 2, 0)
    assert [p.donor for p in pieces] == [0, 1]
    assert all(p.rows == 64 and p.cols == 8 and p.src_ld == 8 and p.dst_ld == 16 for p in pieces)


def test_split_rows_covers_the_run():
    p = Piece(0, 5, 103, 11, 103, 1, 103)
    parts = split_rows(p, limit=10)
    covered = []
    for q in parts:
        for r in range(q.rows):
            covered.extend(range(q.dst_off + r * q.dst_ld, q.dst_off + r * q.dst_ld + q.cols))
    assert covered == list(range(11, 114))
