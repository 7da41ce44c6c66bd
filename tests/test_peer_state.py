"""Peer-state kernels (csrc/peer_state.cu): fused DP all-reduce + AdamW, reshard gather.

Single GPU: the DP kernel runs as group rank 0 of two with the peer's region emulated by
a second region on the same device (its "arrived" flags preset, so no wait is real);
results must equal the sum followed by the stand-alone AdamW kernel bit for bit, and an
FP32 torch AdamW within rounding. The gather kernel moves shards between local regions
and must reproduce ``local_slice`` exactly, plus the bf16 compute copy.

Two GPUs: a DP2 training run through the fused step equals, bit for bit, the same run
with NCCL all-reduce + AdamW (for two ranks both sums are ``g0 + g1``).
"""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu

from resihp.models.layout import TensorSpec  # noqa: E402
from resihp.parallel.tp import FlatState, local_slice  # noqa: E402


def _flat(shapes, device):
    entries = [(TensorSpec(f"t{i}", s, None, "normal"), s) for i, s in enumerate(shapes)]
    return FlatState(entries, device, torch.bfloat16, shared=True)


def test_dp_kernel_matches_sum_then_adamw():
    from resihp.ops import _ext, check_device_errors
    from resihp.ops import functional as fn

    k = _ext.require()
    dev = torch.device("cuda", 0)
    shapes = [(1000, 3), (257,), (4096, 64)]
    a, b = _flat(shapes, dev), _flat(shapes, dev)
    g = torch.Generator(device="cuda").manual_seed(7)
    for f in (a, b):
        for buf in (f.master, f.exp_avg, f.grads[0]):
            buf.copy_(torch.randn(buf.shape, device=dev, generator=g))
        f.exp_avg_sq.copy_(torch.rand(f.numel, device=dev, generator=g))
    b.master.copy_(a.master)
    b.exp_avg.copy_(a.exp_avg)
    b.exp_avg_sq.copy_(a.exp_avg_sq)
    hp = dict(lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1)
    ref_p, ref_m, ref_v = a.master.clone(), a.exp_avg.clone(), a.exp_avg_sq.clone()
    ref_bf = torch.empty_like(a.work)
    total = a.grads[0] + b.grads[0]
    step = 3
    fn.adamw_flat(ref_p, total, ref_m, ref_v, step, lr=hp["lr"], beta1=hp["beta1"], beta2=hp["beta2"], eps=hp["eps"],
                  weight_decay=hp["weight_decay"], p_bf16=ref_bf)
    cpu = [x.cpu() for x in (a.master, a.exp_avg, a.exp_avg_sq)]
    fn.adamw_flat(*cpu[:1], total.cpu(), *cpu[1:], step, lr=hp["lr"], beta1=hp["beta1"], beta2=hp["beta2"],
                  eps=hp["eps"], weight_decay=hp["weight_decay"])
    grid = k.dp_grid(a.numel, 0)
    epoch = 5
    a.flags.view(-1, 8)[:grid, 1] = epoch  # the emulated peer has arrived
    k.dp_allreduce_adamw([a.grads[0].data_ptr(), b.grads[0].data_ptr()], 0, a.grads[1], a.master, a.exp_avg,
                         a.exp_avg_sq, a.work, hp["lr"], hp["beta1"], hp["beta2"], hp["eps"], hp["weight_decay"], step,
                         1.0, a.region_ptr, [a.region_ptr, b.region_ptr], epoch, grid)
    torch.cuda.synchronize()
    check_device_errors(0)
    assert torch.equal(a.grads[1], total)
    assert torch.equal(a.master, ref_p) and torch.equal(a.exp_avg, ref_m) and torch.equal(a.exp_avg_sq, ref_v)
    assert torch.equal(a.work, ref_bf)
    assert torch.equal(b.flags.view(-1, 8)[:grid, 0].cpu(), torch.full((grid,), epoch, dtype=torch.int32))
    torch.testing.assert_close(a.master.cpu(), cpu[0], rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(a.exp_avg_sq.cpu(), cpu[2], rtol=1e-6, atol=0)


def test_dp_push_kernel_matches_sum_then_adamw():
    """The two-phase variant (groups of three and more), run as group rank 0 of three
    with the peers emulated by local regions: every flag a peer would set is preset, and
    the parts the peers would push are preset in this rank's receiving buffer. Rank 0
    must reduce exactly its part of every CTA slice (in rank order), push it into every
    peer's receiving buffer and nowhere else, and step like sum-then-AdamW bit for bit."""
    from resihp.ops import _ext, check_device_errors
    from resihp.ops import functional as fn

    k = _ext.require()
    dev = torch.device("cuda", 0)
    shapes = [(1000, 3), (257,), (4096, 64)]
    regions = [_flat(shapes, dev) for _ in range(3)]
    a = regions[0]
    g = torch.Generator(device="cuda").manual_seed(11)
    for f in regions:
        f.grads[0].copy_(torch.randn(f.numel, device=dev, generator=g))
        f.grads[1].zero_()
    a.master.copy_(torch.randn(a.numel, device=dev, generator=g))
    a.exp_avg.copy_(torch.randn(a.numel, device=dev, generator=g))
    a.exp_avg_sq.copy_(torch.rand(a.numel, device=dev, generator=g))
    total = regions[0].grads[0] + regions[1].grads[0] + regions[2].grads[0]
    a.grads[1].copy_(total)  # the parts the peers push
    hp = dict(lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1)
    ref_p, ref_m, ref_v = a.master.clone(), a.exp_avg.clone(), a.exp_avg_sq.clone()
    ref_bf = torch.empty_like(a.work)
    step, epoch = 2, 7
    fn.adamw_flat(ref_p, total, ref_m, ref_v, step, lr=hp["lr"], beta1=hp["beta1"], beta2=hp["beta2"], eps=hp["eps"],
                  weight_decay=hp["weight_decay"], p_bf16=ref_bf)
    grid = k.dp_grid(a.numel, 0)
    a.flags.view(-1, 8)[:grid, 1:3] = epoch             # phase 0: both peers' gradients are final
    a.flags.view(-1, 8)[grid:2 * grid, 1:3] = epoch     # phase 1: both peers have pushed their parts
    f2 = 4 * 8 * grid
    k.dp_allreduce_adamw([r.grads[0].data_ptr() for r in regions], 0, a.grads[1], a.master, a.exp_avg, a.exp_avg_sq,
                         a.work, hp["lr"], hp["beta1"], hp["beta2"], hp["eps"], hp["weight_decay"], step, 1.0,
                         a.region_ptr, [r.region_ptr for r in regions], epoch, grid,
                         sums_peer=[r.grads[1].data_ptr() for r in regions], flags2_local=a.region_ptr + f2,
                         flags2_peer=[r.region_ptr + f2 for r in regions])
    torch.cuda.synchronize()
    check_device_errors(0)
    assert torch.equal(a.grads[1], total)
    assert torch.equal(a.master, ref_p) and torch.equal(a.exp_avg, ref_m) and torch.equal(a.exp_avg_sq, ref_v)
    assert torch.equal(a.work, ref_bf)
    # rank 0's part of each CTA slice (float4 units), pushed to both peers and only there
    n4 = a.numel // 4
    per = (n4 + grid - 1) // grid
    mine = torch.zeros(n4, dtype=torch.bool)
    for b in range(grid):
        lo, hi = b * per, min(b * per + per, n4)
        if lo >= hi:
            continue
        part = (hi - lo + 2) // 3
        mine[lo:min(lo + part, hi)] = True
    mine = mine.repeat_interleave(4).to(dev)
    for r in regions[1:]:
        assert torch.equal(r.grads[1][mine], total[mine])
        assert torch.count_nonzero(r.grads[1][~mine]) == 0
        assert torch.equal(r.flags.view(-1, 8)[:grid, 0].cpu(), torch.full((grid,), epoch, dtype=torch.int32))
        assert torch.equal(r.flags.view(-1, 8)[grid:2 * grid, 0].cpu(), torch.full((grid,), epoch, dtype=torch.int32))


def test_dp_kernel_reports_a_peer_that_never_arrives():
    """Failure detection on the device, with no fault: the emulated DP peer never flags
    its gradients, the per-launch wait budget is short (50 ms), and the kernel gives up,
    records the peer-wait code and returns without touching the state; the host turns
    the code into a :class:`KernelError`, and the same context runs the kernel
    correctly afterwards."""
    import time

    from resihp.ops import KernelError, _ext, check_device_errors

    k = _ext.require()
    dev = torch.device("cuda", 0)
    a, b = _flat([(4096, 64)], dev), _flat([(4096, 64)], dev)
    a.grads[0].fill_(1.0)
    b.grads[0].fill_(2.0)
    a.master.fill_(0.5)
    before = a.master.clone()
    grid = k.dp_grid(a.numel, 0)
    args = lambda epoch: ([a.grads[0].data_ptr(), b.grads[0].data_ptr()], 0, a.grads[1], a.master, a.exp_avg,  # noqa: E731
                          a.exp_avg_sq, a.work, 1e-3, 0.9, 0.95, 1e-8, 0.0, 1, 1.0, a.region_ptr,
                          [a.region_ptr, b.region_ptr], epoch, grid)
    check_device_errors(0)
    default = k.peer_wait_budget_ns()
    k.set_peer_wait_budget_ns(50_000_000)
    try:
        t0 = time.perf_counter()
        k.dp_allreduce_adamw(*args(9))  # nothing ever sets the peer's epoch-9 flag
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
    finally:
        k.set_peer_wait_budget_ns(default)
    with pytest.raises(KernelError) as info:
        check_device_errors(0)
    assert info.value.code == 4 and "peer" in str(info.value)
    assert 0.04 <= waited < 3.0, waited  # gave up after its budget, not the 4 s default
    assert torch.equal(a.master, before)  # the step did not run
    check_device_errors(0)  # the word was cleared by the read

    a.flags.view(-1, 8)[:grid, 1] = 10  # now the peer has arrived
    k.dp_allreduce_adamw(*args(10))
    torch.cuda.synchronize()
    check_device_errors(0)
    assert torch.equal(a.grads[1], torch.full_like(a.grads[1], 3.0))


def test_reshard_gather_reproduces_local_slices():
    from resihp.ops import check_device_errors
    from resihp.parallel.peer import GatherPlan, shard_pieces

    dev = torch.device("cuda", 0)
    logical = [((512, 96), 0), ((96, 512), 1), ((96,), None), ((200, 70), 1), ((333,), None)]
    fulls = {f"t{i}": {f: torch.randn(s, device=dev) for f in ("param", "exp_avg", "exp_avg_sq")}
             for i, (s, _d) in enumerate(logical)}
    dims = {f"t{i}": d for i, (_s, d) in enumerate(logical)}

    def entries(degree, idx):
        out = []
        for i, (s, d) in enumerate(logical):
            spec = TensorSpec(f"t{i}", s, d, "normal")
            out.append((spec, tuple(local_slice(torch.empty(s), d, idx, degree).shape)))
        return out

    for old, new in ((2, 1), (1, 2), (2, 4), (4, 2)):
        if any(d is not None and s[d] % max(old, new) for s, d in logical):
            continue
        donors = []
        for i in range(old):
            f = FlatState(entries(old, i), dev, torch.bfloat16, shared=True)
            for name, fields in fulls.items():
                d = dims[name]
                f.view(f.master, name).copy_(local_slice(fields["param"], d, i, old))
                f.view(f.exp_avg, name).copy_(local_slice(fields["exp_avg"], d, i, old))
                f.view(f.exp_avg_sq, name).copy_(local_slice(fields["exp_avg_sq"], d, i, old))
            donors.append(f)
        for t in range(new):
            target = FlatState(entries(new, t), dev, torch.bfloat16, shared=True)
            gp = GatherPlan()
            for i, (s, d) in enumerate(logical):
                name = f"t{i}"
                for piece in shard_pieces(s, d, old, new, t):
                    src = donors[piece.donor]
                    gp.add([piece], src_region=src.region_ptr, src_fields=src.field_offsets,
                           src_tensor_off=src.offsets[name][0], dst_flat=target, dst_tensor_off=target.offsets[name][0])
            gp.launch(dev)
            torch.cuda.synchronize()
            check_device_errors(0)
            for i, (s, d) in enumerate(logical):
                name = f"t{i}"
                want = {f: local_slice(fulls[name][f], d, t, new) for f in ("param", "exp_avg", "exp_avg_sq")}
                assert torch.equal(target.view(target.master, name), want["param"]), (old, new, t, name)
                assert torch.equal(target.view(target.exp_avg, name), want["exp_avg"])
                assert torch.equal(target.view(target.exp_avg_sq, name), want["exp_avg_sq"])
                assert torch.equal(target.view(target.work, name), want["param"].bfloat16())


def _dp_worker(rank, world, port, out):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist

    from resihp.config import TrainConfig
    from resihp.control import ControlPlane
    from resihp.ops import check_device_errors
    from resihp.parallel import peer
    from resihp.plan import build_plan
    from resihp.recovery import initial_run

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    store = dist.TCPStore("127.0.0.1", port + 1, world_size=world, is_master=rank == 0, wait_for_workers=False)
    config = TrainConfig(model_dim=256, num_layers=2, num_heads=4, batch_size=8, micro_batch_size=2, seed=3, tp=1,
                         pp=1, dp=world, iterations=4, arch="llama", vocab_size=1024, seq_len=128, ffn_dim=688,
                         dtype="bf16", lr=1e-3, beta1=0.9, beta2=0.95, weight_decay=0.1)
    cp = ControlPlane(rank, range(world), store, "nccl", device=device)  # NCCL groups split from the world
    cp.form_world(range(world), epoch=0)
    plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    groups = cp.build_training_groups(plan)
    results = {}
    for fused in (True, False):
        peer.ENABLED = fused
        run = initial_run(plan, rank=rank, groups=groups, device=device)
        assert (run.runtime.reducer.fused_dp is not None) == fused
        losses = [run.step() for _ in range(3)]
        torch.cuda.synchronize()
        check_device_errors(rank)
        results[fused] = dict(master=run.stage.flat.master.cpu(), exp_avg_sq=run.stage.flat.exp_avg_sq.cpu(),
                              work=run.stage.flat.work.cpu(), grad=run.stage.flat.grad.cpu(), losses=losses)
        run.stage.close_comm()
        del run
    torch.save(results, os.path.join(out, f"dp_{rank}.pt"))
    cp.destroy_training_groups()
    dist.barrier(group=cp.world_group)
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_dp_step_equals_nccl_path(tmp_path):
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_dp_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for rank in range(2):
        r = torch.load(tmp_path / f"dp_{rank}.pt")
        for key in ("master", "exp_avg_sq", "work", "grad"):
            assert torch.equal(r[True][key], r[False][key]), (rank, key)
    a, b = (torch.load(tmp_path / f"dp_{r}.pt")[True]["master"] for r in range(2))
    assert torch.equal(a, b)  # the replicas stay identical
