"""Consistent stops under host-side fault injection (CPU/Gloo, real processes).

* a checkpoint corrupted right after its commit -> every survivor raises
  ``checkpoint_unusable`` at the next safe point;
* one rank planning differently -> every survivor raises ``plan_disagreement``;
* a live replicated weight tampered on a donor right after the commit -> the moved
  state no longer equals the checkpoint (principle A1) -> ``state_mismatch``
  (the reference's fault injector, ``tests/test_recovery.py:455-488``).
Both leave no process group behind and exit cleanly.
"""

import os
from pathlib import Path

import pytest

from harness import assert_killed, read_results, run_ranks, write_result

CONFIG = dict(model_dim=32, num_layers=2, num_heads=4, batch_size=4, micro_batch_size=2, seed=2, tp=2, pp=1, dp=2,
              iterations=4, arch="llama", vocab_size=32, seq_len=8, ffn_dim=64)


def _entry(rank, env, mode, out_dir):
    os.environ.update(env)
    import torch

    torch.set_num_threads(1)
    from resihp import control as control_mod
    from resihp.config import TrainConfig
    from resihp.control import ConsistentStop, ControlPlane
    from resihp.plan import build_plan
    from resihp.recovery import initial_run
    from resihp.train import fail_stop

    config = TrainConfig(**CONFIG)
    cp = ControlPlane.initialize(training_backend="gloo")
    plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    groups = cp.build_training_groups(plan)
    ck = Path(out_dir, "checkpoint.pt")
    cp.attach_run(initial_run(plan, rank=rank, groups=groups), checkpoint_path=ck)
    if mode == "disagree" and rank == 0:
        real = control_mod.build_plan

        def skewed(*a, **k):
            p = real(*a, **k)
            from dataclasses import replace

            return replace(p, step=p.step + 1)

        control_mod.build_plan = skewed
    result = {"rank": rank, "stopped": None}
    failed = ()
    try:
        for it in range(1, config.iterations + 1):
            cp.training_step()
            cp.commit_checkpoint(plan, cursor=it)
            if mode == "corrupt" and it == 2 and rank == 0:
                import torch as t

                cp.flush_checkpoint()  # the writer's background write must be on disk first
                payload = t.load(ck, weights_only=False)
                payload["params"]["final_norm.weight"] = payload["params"]["final_norm.weight"] + 1
                t.save(payload, ck)
            if mode == "tamper" and it == 2 and rank == 0:
                import torch as t

                with t.no_grad():
                    st = cp.training_run.stage
                    st.flat.view(st.flat.master, "final_norm.weight").add_(1.0)
            fail_stop({2: 3}, rank, it)
            lost = cp.observe()
            if lost:
                plan, failed = cp.safe_point(config, plan, failed, lost, next_step=it)
    except ConsistentStop as stop:
        result["stopped"] = stop.reason.code
        import torch.distributed as dist

        result["groups_left"] = cp.groups.tp is not None or bool(cp.groups.hops) or cp.groups.executor is not None
        cp.shutdown()
        result["initialized"] = dist.is_initialized()
        write_result(out_dir, rank, result)
        return
    cp.shutdown()
    write_result(out_dir, rank, result)


@pytest.mark.slow
@pytest.mark.parametrize("mode,code", [("corrupt", "checkpoint_unusable"), ("disagree", "plan_disagreement"),
                                       ("tamper", "state_mismatch")])
def test_consistent_stop(mode, code, tmp_path):
    codes = run_ranks(_entry, 4, mode, str(tmp_path))
    assert_killed(codes, [3], mode)
    results = read_results(tmp_path, [0, 1, 2])
    for r in results.values():
        assert r["stopped"] == code, r
        assert r["groups_left"] is False and r["initialized"] is False
