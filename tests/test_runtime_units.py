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


def test_dp_peers_step_passes_the_right_buffers(monkeypatch):
    """The fused DP step's host side: which gradient parity it reads, where the sum goes,
    the flag arrays, the AdamW step count and the parity swap afterwards."""
    from resihp.ops import _ext
    from resihp.parallel import peer

    class Stub:
        calls = []

        def symm_region(self, total, device):
            return torch.zeros(total, dtype=torch.uint8), b"h"

        def dp_allreduce_adamw(self, *args, **kwargs):
            self.calls.append(args + (kwargs,))

    stub = Stub()
    monkeypatch.setattr(_ext, "require", lambda: stub)
    entries = [(TensorSpec("w", (8, 8), None, "normal"), (8, 8))]
    flat = FlatState(entries, "cpu", torch.bfloat16, shared=True)

    class Stage:
        pass

    stage = Stage()
    stage.flat = flat
    stage.config = _config(dtype="bf16")
    stage.use_grad = flat.set_parity
    dp = peer.DpPeers.__new__(peer.DpPeers)
    dp.rank, dp.bases, dp.grid, dp.epoch, dp.closed, dp.push = 1, [1000, flat.region_ptr], 3, 0, False, False
    for expected_parity in (0, 1, 0):
        assert flat.parity == expected_parity
        dp.step(stage)
        args = stub.calls[-1]
        grads, me, sum_out = args[0], args[1], args[2]
        off = flat.field_offsets[f"grad{expected_parity}"]
        assert grads == [1000 + off, flat.region_ptr + off] and me == 1
        assert sum_out is flat.grads[1 - expected_parity]
        assert args[3] is flat.master and args[4] is flat.exp_avg and args[5] is flat.exp_avg_sq
        assert args[6] is flat.work
        assert args[12] == flat.step and args[14] == flat.region_ptr and args[15] == [1000, flat.region_ptr]
        assert args[16] == dp.epoch and args[17] == 3 and args[18] == {}
    assert flat.step == 3 and flat.parity == 1
    # groups of three and more take the two-phase kernel: the peers' receiving buffers
    # (the sum parity) and the second flag array, right after the first
    dp.push = True
    dp.step(stage)
    extra = stub.calls[-1][18]  # the step read grad1 (parity 1) and sums into grad0
    assert extra["sums_peer"] == [1000 + flat.field_offsets["grad0"], flat.region_ptr + flat.field_offsets["grad0"]]
    assert extra["flags2_local"] == flat.region_ptr + 4 * peer.MAX_DP * 3
    assert extra["flags2_peer"] == [1000 + 4 * peer.MAX_DP * 3, flat.region_ptr + 4 * peer.MAX_DP * 3]


def test_symmetric_workspace_counter_bases_follow_the_kernel(monkeypatch):
    """The fused TP workspace's host bookkeeping: each call passes its epoch, the
    buffers of this epoch's parity on every rank, and the claim counters' bases as they
    stood before the call; the bases then grow by the kernel module's own claim counts
    (AG on its pair of counters, RS and AR on theirs)."""
    import contextlib

    from resihp.ops import _ext
    from resihp.parallel import fused

    class Stub:
        def __init__(self):
            self.ag, self.rs = [], []

        def symm_region(self, total, device):
            return torch.zeros(total, dtype=torch.uint8), b"h"

        def symm_open(self, handle):
            return 1 << 30

        def fused_grid(self, t, n, tp):
            return 7

        def fused_slices(self, rows_per_rank):
            return 16

        def fused_tile_claims(self, t, n, grid):
            return 100 + grid

        def fused_copy_claims(self, mode, t, n, tp, slices, xg, grid):
            return {1: 50 if xg else 20, 2: 15, 3: 30}[mode] + grid

        def ag_gemm(self, x_local, xg, w, w_mn, y, peers, grid):
            self.ag.append((xg, peers, grid))

        def gemm_rs(self, h, w, w_mn, y, all_reduce, peers, grid):
            self.rs.append((y.shape, all_reduce, peers))

    stub = Stub()
    monkeypatch.setattr(_ext, "require", lambda: stub)
    monkeypatch.setattr(fused.dist, "get_world_size", lambda group: 4)
    monkeypatch.setattr(fused.dist, "get_rank", lambda group: 1)
    monkeypatch.setattr(fused.dist, "all_gather_object", lambda out, obj, group: out.__setitem__(slice(None), [obj] * 4))
    monkeypatch.setattr(fused.dist, "barrier", lambda group=None: None)
    monkeypatch.setattr(torch.cuda, "device", lambda d: contextlib.nullcontext())
    monkeypatch.setattr(torch.cuda, "synchronize", lambda d=None: None)
    ws = fused.SymmetricWorkspace(None, 128, 64, "cpu")
    tp = 4
    peers_of = [1 << 30, ws.base, 1 << 30, 1 << 30]  # this rank is group rank 1
    assert ws.slices == 16 and ws.t == 512
    x = torch.zeros(128, 64, dtype=torch.bfloat16)
    w = torch.zeros(32, 64, dtype=torch.bfloat16)
    for call in range(1, 4):
        ws.all_gather_gemm(x, w, False, 32)
        xg, peers, grid = stub.ag[-1]
        assert xg is not None and tuple(xg.shape) == (512, 64) and grid == 7
        assert peers[:6] == [1, tp, 128, 16, call, 0]                      # rank, tp, rows, slices, epoch, ar epoch
        assert peers[6] == ws.base + fused._CTRS and peers[7] == (107 * (call - 1))      # AG tile counter, base
        assert peers[8] == ws.base + fused._CTRS + 4 and peers[9] == (57 * (call - 1))   # AG copy counter, base
        land = peers[10:10 + tp]
        assert land == [b + ws.land_off + (call % 2) * ws.stride for b in peers_of]
        assert peers[10 + tp:10 + 2 * tp] == [b + fused._AG_CNT for b in peers_of]
    ws.all_gather_gemm(x, w, False, 32, keep_gathered=False)
    assert stub.ag[-1][0] is None and stub.ag[-1][1][9] == 57 * 3
    assert ws.bases[1] == 57 * 3 + 27                                         # no gathered copy: fewer items
    h = torch.zeros(512, 16, dtype=torch.bfloat16)
    ws.gemm_reduce_scatter(h, torch.zeros(64, 16, dtype=torch.bfloat16), False, 64)
    shape, ar, peers = stub.rs[-1]
    assert tuple(shape) == (128, 64) and not ar and peers[4] == 1 and peers[5] == 0
    assert peers[7] == 0 and peers[9] == 0                                    # RS counters start fresh
    assert peers[10 + 2 * tp:10 + 3 * tp] == [b + ws.recv_off + ws.stride for b in peers_of]
    ws.gemm_all_reduce(h, torch.zeros(64, 16, dtype=torch.bfloat16), False, 64)
    shape, ar, peers = stub.rs[-1]
    assert tuple(shape) == (512, 64) and ar and peers[4] == 2 and peers[5] == 1
    assert peers[7] == 107 and peers[9] == 22                                 # after one RS
    assert peers[10 + 4 * tp:10 + 5 * tp] == [b + ws.out_off + ws.stride for b in peers_of]
    assert peers[10 + 5 * tp:10 + 6 * tp] == [b + fused._AR_CNT for b in peers_of]
    assert peers[10 + 6 * tp:] == [ws.base + ws.send_off, ws.base + fused._SEND_CNT, ws.base + fused._OWN_CNT]
    assert ws.bases == [107 * 4, 57 * 3 + 27, 107 * 2, 22 + 37]


def test_control_plane_run_constants_must_match_the_config():
    """The reference's ``ControlPlane(vocab_size=, sequence_length=)`` is accepted; a value
    that disagrees with the config stops the safe point before any collective."""
    from resihp.control import ControlPlane

    config = TrainConfig(model_dim=16, num_layers=2, num_heads=2, batch_size=2, micro_batch_size=1, seed=1, tp=1,
                         pp=2, dp=1, iterations=2, vocab_size=32, seq_len=8)
    plan = build_plan(config, step=0, version=0, vocab_size=32, sequence_length=8)
    cp = ControlPlane(0, range(2), None, "gloo", vocab_size=64, sequence_length=8)
    assert (cp.vocab_size, cp.sequence_length) == (64, 8)
    with pytest.raises(ValueError, match="vocab_size=64 does not match the config"):
        cp.safe_point(config, plan, (), (1,), next_step=1)


def test_trace_categories_name_the_linear_layer_products():
    from resihp.utils.trace import categorize

    rows = [
        {"name": "void resihp::gemm_kernel<256, false, false, 0>(CUtensorMap_st, CUtensorMap_st, resihp::GemmArgs)",
         "calls": 10, "device_us": 600.0},
        {"name": "_ZN6resihp11gemm_kernelILi256ELb1ELb1ELi2EEEv14CUtensorMap_stS1_NS_8GemmArgsE", "calls": 5,
         "device_us": 300.0},
        {"name": "void resihp::gemm_kernel<128, false, true, 0>(...)", "calls": 2, "device_us": 50.0},
        {"name": "void resihp::fused_gemm_kernel<256, false, 1, 0>(...)", "calls": 1, "device_us": 20.0},
        {"name": "void resihp::(anonymous namespace)::attn_bwd_dq_kernel<128>(...)", "calls": 1, "device_us": 20.0},
        {"name": "ncclDevKernel_AllReduce_Sum_f32_RING_LL(...)", "calls": 1, "device_us": 5.0},
        {"name": "void at::native::vectorized_elementwise_kernel<4>(...)", "calls": 1, "device_us": 5.0},
    ]
    cats = categorize(rows)
    assert list(cats)[:2] == ["GEMM forward", "GEMM wgrad"]
    # the CTA-pair GEMM, the vector elementwise kernels and the two-phase DP step
    more = categorize([
        {"name": "void resihp::gemm_pair_kernel<false, true, 0, 6>(CUtensorMap_st, CUtensorMap_st, resihp::GemmArgs)",
         "calls": 3, "device_us": 30.0},
        {"name": "_ZN6resihp16gemm_pair_kernelILb1ELb1ELi4ELi6EEEv14CUtensorMap_stS1_NS_8GemmArgsE", "calls": 2,
         "device_us": 20.0},
        {"name": "resihp::(anonymous namespace)::rope_vec_kernel(__nv_bfloat16*, ...)", "calls": 1, "device_us": 4.0},
        {"name": "resihp::(anonymous namespace)::adamw_vec_kernel(float4*, ...)", "calls": 1, "device_us": 3.0},
        {"name": "void resihp::dp_adamw_push_kernel<2>(...)", "calls": 1, "device_us": 2.0},
        {"name": "resihp::(anonymous namespace)::embedding_sort_kernel(long const*, ...)", "calls": 1,
         "device_us": 1.0},
    ])
    assert more["GEMM dgrad"]["calls"] == 3 and more["GEMM wgrad"]["calls"] == 2
    assert more["RoPE / SwiGLU / embedding"]["calls"] == 2 and more["AdamW"]["calls"] == 1
    assert more["fused DP all-reduce + AdamW"]["calls"] == 1 and "other" not in more
    assert cats["GEMM dgrad"]["calls"] == 2 and cats["fused TP collective GEMM"]["device_us"] == 20.0
    assert cats["attention backward"]["share"] == 0.02 and cats["NCCL"]["calls"] == 1 and "other" in cats
    assert abs(sum(c["share"] for c in cats.values()) - 1.0) < 1e-3
