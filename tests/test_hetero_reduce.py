"""The P2P heterogeneous-replica gradient sum, executed on host buffers.

After a fail-stop the replicas can hold the same logical tensor at different TP degrees
and layer placements (and, with tied embeddings, twice per replica). The P2P reduction
(:class:`resihp.parallel.peer.HeteroPeers`) has every rank pull the pieces of the other
holders' gradients of its own shards and add the holders' contributions in (replica,
stage) order. Here every rank's flat state is a host buffer; the copy descriptors are
executed by a host interpreter of the gather kernel and the ordered sums are compared
with the logical definition -- the sum over holder stages of each stage's full
gradient, sliced to the rank's shard -- and across ranks that hold the same elements.
"""

import ctypes

import pytest
import torch

from resihp.config import TrainConfig
from resihp.models.layout import local_shape, model_specs, stage_specs
from resihp.ops import _ext
from resihp.parallel import peer
from resihp.parallel.tp import FlatState, local_slice
from resihp.plan import build_plan
from resihp.recovery import stage_ends, stage_layout, stage_of


class _HostRegions:
    def __init__(self):
        self.keep = []

    def symm_region(self, total, device):
        t = torch.zeros(total, dtype=torch.uint8)
        self.keep.append(t)
        return t, b"host"


def _plan(failed, **kw):
    base = dict(model_dim=64, num_layers=6, num_heads=4, batch_size=8, micro_batch_size=2, seed=1, tp=2, pp=2, dp=2,
                iterations=4, arch="llama", vocab_size=64, seq_len=16, ffn_dim=96, dtype="bf16")
    base.update(kw)
    config = TrainConfig(**base)
    plan = build_plan(config, step=0, version=0, vocab_size=64, sequence_length=16)
    seen = []
    for i, r in enumerate(failed):
        seen.append(r)
        plan = build_plan(config, step=i + 1, version=plan.version + 1, failed_ranks=tuple(seen), previous=plan,
                          vocab_size=64, sequence_length=16)
    return config, plan


def _execute(rows):
    for src, dst, _bf16, src_ld, dst_ld, nrows, cols, _base, _vec4 in rows:
        for r in range(nrows):
            ctypes.memmove(dst + 4 * r * dst_ld, src + 4 * r * src_ld, 4 * cols)


@pytest.mark.parametrize("failed,extra", [((5,), {}), ((5, 2), {"tied_embeddings": True}), ((1,), {"pp": 1})])
def test_p2p_hetero_sum_matches_the_logical_sum(monkeypatch, failed, extra):
    host = _HostRegions()
    monkeypatch.setattr(_ext, "require", lambda: host)
    config, plan = _plan(failed, **extra)
    shapes = {s.name: s.shape for s in model_specs(config)}
    g = torch.Generator().manual_seed(sum(failed))
    flats, metas = {}, {}
    for rank in plan.active_ranks:
        sp = stage_of(plan, rank)
        first, last = stage_ends(plan, sp)
        specs = stage_specs(config, range(*sp.layer_range), first, last)
        flat = FlatState([(s, local_shape(s, sp.tp_degree)) for s in specs], "cpu", torch.bfloat16, shared=True)
        flat.grads[0].copy_(torch.randn(flat.numel, generator=g))
        flats[rank] = flat
        metas[rank] = peer.StageMeta(rank, sp.replica_id, sp.stage_id, tuple(sp.tp_members), stage_layout(plan, sp),
                                     flat.export())
    # replicated tensors: every TP member of a stage holds the stage's (identical) total
    for rank, m in metas.items():
        lead = flats[m.tp_members[0]]
        for name, dim in m.layout.items():
            if dim is None:
                flats[rank].view(flats[rank].grads[0], name).copy_(lead.view(lead.grads[0], name))

    # the logical definition: per holder stage, its full gradient; summed over holders
    stages = {(m.replica, m.stage): m for m in metas.values()}
    want_full = {}
    for name in shapes:
        total = torch.zeros(shapes[name])
        for key in sorted(stages):
            m = stages[key]
            if name not in m.layout:
                continue
            dim = m.layout[name]
            parts = [flats[r].view(flats[r].grads[0], name) for r in m.tp_members]
            total += parts[0] if dim is None else torch.cat(parts, dim=dim)
        want_full[name] = total

    results = {}
    for rank, m in metas.items():
        flat = flats[rank]
        terms = peer.hetero_terms(metas, rank, shapes)
        scratch = torch.zeros((4, flat.numel))
        gather, slots = peer.hetero_gather(terms, metas, rank, flat, lambda r: flats[r].region_ptr, scratch)
        _execute(gather.rows)
        # the sums overwrite this rank's gradients: the other ranks' pulls above read the
        # originals, so sum into a copy and compare
        grad = flat.grads[0].clone()
        peer.hetero_sum(terms, slots, scratch, flat, grad)
        idx = m.tp_members.index(rank)
        for name, _own, _pieces in terms:
            acc = flat.view(grad, name)
            want = local_slice(want_full[name], m.layout[name], idx, len(m.tp_members))
            torch.testing.assert_close(acc, want, rtol=1e-6, atol=1e-6)
            results[(rank, name)] = (m.layout[name], idx, len(m.tp_members), acc)

    # ranks holding the same elements computed the same bits
    for (r1, name), (dim, i1, d1, a1) in results.items():
        for (r2, n2), (_d, i2, d2, a2) in results.items():
            if n2 == name and r2 != r1 and d1 == d2 and i1 == i2:
                assert torch.equal(a1, a2), (name, r1, r2)
