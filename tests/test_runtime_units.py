"""Pure pieces of the distributed runtime, checked without a process group.

* pipeline boundary routing (reference ``resihp/parallel/pp.py:73-96``): with
  ``N = max(U, D)`` chunks, chunk ``k`` travels ``up[k U / N] -> down[k D / N]``; every
  chunk is sent once, and each sender / receiver handles a contiguous run of chunks;
* data-parallel executor routes after a reroute, the global micro-batch count and the
  activation log (reference ``resihp/parallel/dp.py:38-95``);
* the reduction topology the control plane builds groups from: homogeneous replicas get
  one DP group per (stage, TP index), heterogeneous ones the logical path, tied
  embeddings one pair per replica and TP index;
* the flat state's gradient parity on the CPU path.
"""

import itertools

import pytest
import torch

from resihp.config import TrainConfig
from resihp.models.layout import TensorSpec
from resihp.parallel.dp import ActivationLog, executor_route, global_micro_count, reduction_topology
from resihp.parallel.pp import scatter_routing
from resihp.parallel.tp import FlatState
from resihp.plan import build_plan
from resihp.recovery import dp_assignment

DEGREES = (1, 2, 4, 8)


def _config(**kw):
    base = dict(model_dim=64, num_layers=4, num_heads=4, batch_size=8, micro_batch_size=2, seed=1, tp=2, pp=2, dp=2,
                iterations=4, arch="llama", vocab_size=64, seq_len=16, ffn_dim=96)
    base.update(kw)
    return TrainConfig(**base)


def _plan(config, failed=()):
    plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    seen = []
    for i, r in enumerate(failed):
        seen.append(r)
        plan = build_plan(config, step=i + 1, version=plan.version + 1, failed_ranks=tuple(seen), previous=plan,
                          vocab_size=config.vocab_size, sequence_length=config.seq_len)
    return plan


@pytest.mark.parametrize("u,d", list(itertools.product(DEGREES, DEGREES)))
def test_scatter_routing_sends_each_chunk_once_contiguously(u, d):
    up = tuple(range(100, 100 + u))
    down = tuple(range(200, 200 + d))
    route = scatter_routing(up, down)
    n = max(u, d)
    assert len(route) == n
    for k, (s, r) in enumerate(route):
        assert s == up[k * u // n] and r == down[k * d // n]
    for members, side in ((up, 0), (down, 1)):
        for m in members:
            ks = [k for k, pair in enumerate(route) if pair[side] == m]
            assert ks and ks == list(range(ks[0], ks[-1] + 1)), (m, ks)
            assert len(ks) == n // len(members)


def test_executor_routes_follow_the_assignment_after_a_reroute():
    config = _config()
    plan = _plan(config, failed=(5,))  # replica 1 loses a stage-0 rank
    assignment = dp_assignment(plan)
    assert global_micro_count(assignment) == config.batch_size // config.micro_batch_size
    executed = {}
    for rank in plan.active_ranks:
        for entry in executor_route(assignment, rank):
            executed.setdefault((entry["micro_batch"], entry["stage_id"]), set()).add(rank)
            assert rank in entry["executors"]
            if entry["upstream"] is None:
                assert entry["stage_id"] == min(p.stage_id for p in assignment.by_micro_batch[entry["micro_batch"]])
            if entry["downstream"] is not None:
                nxt = [e for r2 in entry["downstream"] for e in executor_route(assignment, r2)
                       if e["micro_batch"] == entry["micro_batch"]]
                assert nxt and all(e["upstream"] == entry["executors"] for e in nxt)
    # every micro-batch runs every stage of exactly one replica, exactly once
    for mb, placements in assignment.by_micro_batch.items():
        for p in placements:
            assert executed[(mb, p.stage_id)] == set(p.executor_ranks)


def test_activation_log_peak_and_misuse():
    log = ActivationLog()
    for k in range(3):
        log.retain(k)
    log.release(1)
    log.retain(3)
    assert log.peak == 3 and log.live == {0, 2, 3}
    with pytest.raises(KeyError):
        log.release(7)


def test_reduction_topology_homogeneous_heterogeneous_and_tied():
    config = _config()
    topo = reduction_topology(_plan(config))
    assert topo.homogeneous
    # (stage, tp index) positions across the two replicas: ranks r and r + 4
    assert sorted(topo.dp_groups) == [(0, 4), (1, 5), (2, 6), (3, 7)]
    assert topo.tied_groups == ()
    hetero = reduction_topology(_plan(config, failed=(5,)))
    assert not hetero.homogeneous and hetero.dp_groups == () and hetero.tied_groups == ()
    tied = reduction_topology(_plan(_config(tied_embeddings=True)))
    # embedding stage rank and head stage rank of the same TP index, per replica
    assert sorted(tied.tied_groups) == [(0, 2), (1, 3), (4, 6), (5, 7)]


def test_flat_state_views_and_parity_on_cpu():
    entries = [(TensorSpec("a", (3, 5), 0, "normal"), (3, 5)), (TensorSpec("b", (7,), None, "ones"), (7,))]
    flat = FlatState(entries, "cpu", torch.float32)
    assert flat.numel % 64 == 0 and flat.work is flat.master and len(flat.grads) == 1
    a = flat.view(flat.master, "a")
    a.fill_(2.0)
    assert flat.master[:15].eq(2.0).all() and flat.offsets["b"][0] % 64 == 0
    flat.set_parity(0)
    assert flat.grad is flat.grads[0]
    assert flat.export()["offsets"] == {"a": 0, "b": flat.offsets["b"][0]}


def test_trace_ranges_are_free_when_off():
    from resihp.utils import trace

    with trace.nvtx_range("F0"):
        pass
    assert not trace._ON or torch.cuda.is_available()


def test_disjoint_layers_partition_groups_in_order():
    from resihp.control import ControlPlane

    groups = [(0, 1), (2, 3), (1, 2), (4,), (0, 4), (3, 5)]
    layers = ControlPlane.disjoint_layers(groups)
    assert layers == [[(0, 1), (2, 3), (4,)], [(1, 2), (0, 4), (3, 5)]]
    for layer in layers:
        seen = [r for grp in layer for r in grp]
        assert len(seen) == len(set(seen))
    assert sorted(g for layer in layers for g in layer) == sorted(groups)
