"""Training-group construction reuses the world where a group would equal it (CPU/Gloo).

At a safe point every communicator costs time to create (an ``ncclCommSplit`` each on
GPUs). The executor group spans the plan's active ranks and the live group spans every
member: when those are exactly the world's members, the world group itself serves, and
tearing the training groups down leaves the world alive. Every rank takes the same
decision from the plan, so the collective ``new_group`` calls stay matched.
"""

import os

import pytest

from harness import read_results, run_ranks, write_result

CONFIG = dict(model_dim=32, num_layers=2, num_heads=4, batch_size=4, micro_batch_size=1, seed=2, tp=2, pp=1, dp=2,
              iterations=2, arch="llama", vocab_size=32, seq_len=8, ffn_dim=64)


def _entry(rank, env, out_dir):
    os.environ.update(env)
    import torch

    torch.set_num_threads(1)
    import torch.distributed as dist

    from resihp.config import TrainConfig
    from resihp.control import ControlPlane
    from resihp.plan import build_plan

    config = TrainConfig(**CONFIG)
    cp = ControlPlane.initialize(training_backend="gloo")
    plan = build_plan(config, step=0, version=0, vocab_size=32, sequence_length=8)
    groups = cp.build_training_groups(plan)
    full = {"executor_is_world": groups.executor is cp.world_group, "live_is_world": groups.live is cp.world_group}
    t = torch.ones(1)
    dist.all_reduce(t, group=groups.executor)
    cp.destroy_training_groups()
    dist.barrier(group=cp.world_group)  # the world survived the teardown
    # a plan with rank 3 failed: its active ranks are a strict subset of the members
    smaller = build_plan(config, step=1, version=1, failed_ranks=(3,), previous=plan, vocab_size=32, sequence_length=8)
    groups = cp.build_training_groups(smaller)
    part = {"executor_is_world": groups.executor is cp.world_group, "live_is_world": groups.live is cp.world_group,
            "active": list(smaller.active_ranks)}
    if groups.executor is not None:
        t = torch.ones(1)
        dist.all_reduce(t, group=groups.executor)
        part["executor_sum"] = float(t.item())
    write_result(out_dir, rank, {"full": full, "part": part})
    cp.shutdown()


@pytest.mark.slow
def test_executor_and_live_groups_reuse_the_world(tmp_path):
    codes = run_ranks(_entry, 4, str(tmp_path))
    assert set(codes.values()) == {0}, codes
    results = read_results(tmp_path, range(4))
    for rank, r in results.items():
        assert r["full"] == {"executor_is_world": True, "live_is_world": True}, rank
        assert r["part"]["live_is_world"] is True
        active = r["part"]["active"]
        assert len(active) < 4
        if rank in active:
            assert r["part"]["executor_is_world"] is False and r["part"]["executor_sum"] == float(len(active))
