"""``column_parallel_linear`` on Gloo ranks (FP32): the overlapped backward gives the same
forward, input gradient and weight gradient as the plain column-parallel product, with
and without sequence parallelism."""

import os

import pytest
import torch

from harness import read_results, run_ranks, write_result


def _entry(rank, env, out_dir):
    os.environ.update(env)
    import torch.distributed as dist

    torch.set_num_threads(1)
    from resihp.parallel.collectives import column_parallel_linear

    dist.init_process_group("gloo", init_method=f"tcp://{os.environ['RESIHP_T_ADDR']}", rank=rank, world_size=2)
    d, n, t = 16, 24, 8
    errs = {}
    for sp in (True, False):
        x_full = torch.randn(t, d, generator=torch.Generator().manual_seed(1))
        w = torch.nn.Parameter(torch.randn(n, d, generator=torch.Generator().manual_seed(10 + rank)))
        dy = torch.randn(t, n, generator=torch.Generator().manual_seed(20 + rank))
        x_in = (x_full[rank * t // 2:(rank + 1) * t // 2] if sp else x_full).clone().requires_grad_()
        y = column_parallel_linear(x_in, w, None, dist.group.WORLD, sp)
        y.backward(dy)
        ws = [torch.empty_like(w) for _ in range(2)]
        dys = [torch.empty_like(dy) for _ in range(2)]
        dist.all_gather(ws, w.detach())
        dist.all_gather(dys, dy)
        dx_full = dys[0] @ ws[0] + dys[1] @ ws[1]
        want_dx = dx_full[rank * t // 2:(rank + 1) * t // 2] if sp else dx_full
        errs[f"y{sp}"] = (y.detach() - x_full @ w.detach().t()).abs().max().item()
        errs[f"dx{sp}"] = (x_in.grad - want_dx).abs().max().item()
        errs[f"dw{sp}"] = (w.grad - dy.t() @ x_full).abs().max().item()
    write_result(out_dir, rank, errs)
    dist.destroy_process_group()


@pytest.mark.slow
def test_column_parallel_linear_on_gloo(tmp_path, monkeypatch):
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        monkeypatch.setenv("RESIHP_T_ADDR", f"127.0.0.1:{s.getsockname()[1]}")
    codes = run_ranks(_entry, 2, str(tmp_path))
    assert set(codes.values()) == {0}, codes
    for rank, errs in read_results(tmp_path, [0, 1]).items():
        assert all(v < 1e-4 for v in errs.values()), (rank, errs)
