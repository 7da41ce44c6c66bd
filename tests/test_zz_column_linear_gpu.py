"""The NCCL column-parallel linear with its backward collective overlapped (2+ GPUs, last).

``column_parallel_linear`` (used at TP degrees above the fused-kernel cap) starts the
input gradient's reduce-scatter (SP) or all-reduce asynchronously and computes the
weight gradient while it is in flight. Forward, input gradient and weight gradient
must match an FP32 torch reference of the same column-parallel product, with and
without sequence parallelism. Skipped with fewer than two GPUs.
"""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, out):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    from resihp.ops import check_device_errors
    from resihp.parallel.collectives import column_parallel_linear

    d, n, t = 512, 768, 256 * world
    tl = t // world
    errs = {}
    for sp in (True, False):
        g = torch.Generator(device="cuda").manual_seed(7)
        x_full = torch.randn(t, d, device="cuda", generator=g).bfloat16()
        gr = torch.Generator(device="cuda").manual_seed(100 + rank)
        w = (torch.randn(n, d, device="cuda", generator=gr) / d**0.5).bfloat16().requires_grad_()
        dy = torch.randn(t, n, device="cuda", generator=gr).bfloat16()
        x_in = (x_full[rank * tl:(rank + 1) * tl] if sp else x_full).contiguous().requires_grad_()
        mg = torch.zeros(n, d, device="cuda")
        y = column_parallel_linear(x_in, w, mg, dist.group.WORLD, sp)
        ref = x_full.float() @ w.detach().float().t()
        errs[f"fwd_sp{sp}"] = ((y.float() - ref).norm() / ref.norm()).item()
        y.backward(dy)
        part = (dy.float() @ w.detach().float()).contiguous()  # this rank's partial input gradient
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        ref_dx = sum(parts)[rank * tl:(rank + 1) * tl] if sp else sum(parts)
        errs[f"dx_sp{sp}"] = ((x_in.grad.float() - ref_dx).norm() / ref_dx.norm()).item()
        ref_dw = dy.float().t() @ x_full.float()
        errs[f"dw_sp{sp}"] = ((mg - ref_dw).norm() / ref_dw.norm()).item()
    torch.cuda.synchronize()
    check_device_errors(rank)
    torch.save(errs, os.path.join(out, f"errs_{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_column_parallel_linear_overlapped_backward(tmp_path):
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        errs = torch.load(tmp_path / f"errs_{r}.pt")
        for k, v in errs.items():
            assert v < (1e-3 if k.startswith("dw") else 1.5e-2), (r, k, v, errs)
