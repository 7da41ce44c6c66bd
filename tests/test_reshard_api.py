"""The any-layout reshard and gradient-combine functions (``resihp.parallel.reshard``,
``resihp.parallel.dp.dp_combine_gradients``): pure cases, then real Gloo ranks.

* Reconstruction takes a replicated tensor from any holder, a sharded one only when
  every shard of one degree is present, else the checkpoint, else raises.
* ``reshard_tp_state`` over three ranks re-cuts a TP2 state (plus a stray degree-1
  copy) to a new TP2 group that includes a rank which held nothing, with the donor-only
  rank receiving nothing; checkpoint verification accepts the true state, and every
  rank raises on a corrupted checkpoint and on a tensor with a shard missing everywhere.
* ``dp_combine_gradients`` sums a TP2 replica and a TP1 replica of the same tensors.
"""

import os

import pytest
import torch

from harness import read_results, run_ranks, write_result
from resihp.config import TrainConfig
from resihp.models import layout
from resihp.parallel.reshard import ReshardError, reconstruct_full, shard_dims, shard_logical_state
from resihp.parallel.tp import local_slice

CONFIG = dict(model_dim=16, num_layers=2, num_heads=2, batch_size=2, micro_batch_size=1, seed=5, tp=2, pp=1, dp=1,
              iterations=1, vocab_size=32, seq_len=8)


def _full_state(seed=0):
    config = TrainConfig(**CONFIG)
    g = torch.Generator().manual_seed(seed)
    out = {}
    for s in layout.model_specs(config):
        out[s.name] = {f: torch.randn(s.shape, generator=g) for f in ("param", "exp_avg", "exp_avg_sq")}
        out[s.name]["step"] = torch.tensor(3.0)
    return out


def test_reconstruct_full_cases():
    full = torch.arange(24.0).view(4, 6)
    parts = {i: c for i, c in enumerate(torch.chunk(full, 2, dim=1))}
    assert torch.equal(reconstruct_full("w", 1, 2, parts)[0], full)
    assert reconstruct_full("w", 1, 2, parts)[1] == "peer"
    assert reconstruct_full("n", None, 4, {3: full})[1] == "peer"
    got, source = reconstruct_full("w", 1, 2, {0: parts[0]}, {"w": full})
    assert source == "checkpoint" and torch.equal(got, full)
    with pytest.raises(ReshardError, match="w unavailable"):
        reconstruct_full("w", 1, 2, {0: parts[0]})


def test_shard_dims_and_slicing_follow_the_layout():
    config = TrainConfig(**dict(CONFIG, arch="llama", ffn_dim=32))
    assert shard_dims(range(2), config) == layout.shard_dims(config)
    dims = shard_dims([0, 1])  # GPT-2 names without a config
    assert dims["layers.1.attn.out_proj.weight"] == 1 and dims["position_embedding.weight"] is None
    full = {n: e["param"] for n, e in _full_state().items()}
    cut = shard_logical_state(full, layout=dims, tp_rank=1, tp_size=2)
    for name, dim in dims.items():
        assert torch.equal(cut[name], local_slice(full[name], dim, 1, 2))


def _reshard_entry(rank, env, out_dir):
    os.environ.update(env)
    import torch.distributed as dist

    torch.set_num_threads(1)
    from resihp.parallel.reshard import ReshardError, reshard_tp_state

    dist.init_process_group("gloo", init_method=f"tcp://{os.environ['RESIHP_T_ADDR']}", rank=rank, world_size=3)
    full = _full_state()
    dims = shard_dims([0, 1])
    local = {}
    if rank in (0, 1):  # the old TP2 group
        for name, dim in dims.items():
            local[name] = {"shard_index": rank, **{f: local_slice(t, None if f == "step" else dim, rank, 2)
                                                   for f, t in full[name].items()}}
    if rank == 2:  # a stray full copy of one tensor, cut at degree 1
        local["lm_head.weight"] = {"shard_index": 0, "shard_count": 1, **full["lm_head.weight"]}
    new_rank = {0: 0, 1: None, 2: 1}[rank]
    got = reshard_tp_state(local, layout=dims, old_size=2, new_size=2, new_rank=new_rank, checkpoint=full)
    ok = True
    if new_rank is None:
        ok = got == {}
    else:
        for name, dim in dims.items():
            for f, t in full[name].items():
                ok &= torch.equal(got[name][f], local_slice(t, None if f == "step" else dim, new_rank, 2))
    bad = {n: dict(e) for n, e in full.items()}
    bad["layers.1.mlp.fc2.weight"]["exp_avg"] = bad["layers.1.mlp.fc2.weight"]["exp_avg"] + 1e-3
    try:
        reshard_tp_state(local, layout=dims, old_size=2, new_size=2, new_rank=new_rank, checkpoint=bad)
        caught = None
    except ReshardError as error:
        caught = str(error)
    missing = dict(local)
    if rank == 0:  # one shard of a sharded tensor gone, its partner still held
        missing.pop("layers.0.mlp.fc1.weight")
    try:
        reshard_tp_state(missing, layout=dims, old_size=2, new_size=2, new_rank=new_rank)
        lost = None
    except ReshardError as error:
        lost = str(error)
    write_result(out_dir, rank, {"ok": bool(ok), "caught": caught, "lost": lost})
    dist.destroy_process_group()


def _combine_entry(rank, env, out_dir):
    os.environ.update(env)
    import torch.distributed as dist

    torch.set_num_threads(1)
    from resihp.parallel.dp import dp_combine_gradients

    dist.init_process_group("gloo", init_method=f"tcp://{os.environ['RESIHP_T_ADDR']}", rank=rank, world_size=3)
    a, b = _full_state(1), _full_state(2)
    dims = shard_dims([0, 1])
    replica, degree, index = {0: (0, 2, 0), 1: (0, 2, 1), 2: (1, 1, 0)}[rank]
    source = a if replica == 0 else b
    local = {n: {"grad": local_slice(source[n]["param"], d, index, degree), "shard_dim": d, "shard_index": index,
                 "old_size": degree, "replica": replica} for n, d in dims.items()}
    got = dp_combine_gradients(local)
    ok = all(torch.equal(got[n], local_slice(a[n]["param"] + b[n]["param"], d, index, degree))
             for n, d in dims.items())
    write_result(out_dir, rank, {"ok": bool(ok)})
    dist.destroy_process_group()


def _addr():
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return f"127.0.0.1:{s.getsockname()[1]}"


@pytest.mark.slow
def test_reshard_tp_state_over_gloo_ranks(tmp_path, monkeypatch):
    monkeypatch.setenv("RESIHP_T_ADDR", _addr())
    codes = run_ranks(_reshard_entry, 3, str(tmp_path))
    assert set(codes.values()) == {0}, codes
    for rank, r in read_results(tmp_path, range(3)).items():
        assert r["ok"], rank
        assert r["caught"] == "reshard verify failed for layers.1.mlp.fc2.weight.exp_avg", r
        assert r["lost"] == "logical tensor layers.0.mlp.fc1.weight unavailable from peers and checkpoint", r


@pytest.mark.slow
def test_dp_combine_gradients_across_degrees(tmp_path, monkeypatch):
    monkeypatch.setenv("RESIHP_T_ADDR", _addr())
    codes = run_ranks(_combine_entry, 3, str(tmp_path))
    assert set(codes.values()) == {0}, codes
    assert all(r["ok"] for r in read_results(tmp_path, range(3)).values())
