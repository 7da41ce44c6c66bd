"""Process entry points of the distributed CPU/Gloo gates (importable by spawned children)."""

import json
import os
import sys
from pathlib import Path

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _setup(env):
    os.environ.update(env)
    import faulthandler

    import torch

    torch.set_num_threads(1)
    # a rank stuck in a collective prints every thread's stack instead of hanging silently
    faulthandler.dump_traceback_later(240, repeat=True)


def train_entry(rank, env, config_dict, steps, out_dir, dump_state):
    """Train ``steps`` iterations of one plan; write losses (+ final shards) per rank."""
    _setup(env)
    import torch

    from harness import write_result
    from resihp.config import TrainConfig
    from resihp.control import ControlPlane
    from resihp.plan import build_plan
    from resihp.recovery import initial_run

    config = TrainConfig(**config_dict)
    cp = ControlPlane.initialize(training_backend="gloo")
    plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    groups = cp.build_training_groups(plan)
    run = initial_run(plan, rank=rank, groups=groups)
    losses = []
    for _ in range(steps):
        losses.append(run.step() if run is not None else None)
    result = {"rank": rank, "losses": losses, "schedule": None if run is None else run.runtime.schedule}
    if dump_state and run is not None:
        shards = {n: t.detach().tolist() for n, (t, _d) in run.stage.local_shards().items()}
        result.update(shards=shards, tp_rank=run.stage.tp_rank, tp_size=run.stage.tp_size)
    write_result(out_dir, rank, result)
    cp.shutdown()


def _device(gpu):
    """This rank's GPU (``LOCAL_RANK``) for the GPU variants of the gates, else the CPU."""
    import torch

    if not gpu:
        return None, "gloo"
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    return torch.device("cuda", torch.cuda.current_device()), "nccl"


def failstop_entry(rank, env, config_dict, failures, out_dir, gpu=False):
    """The worker loop with a failure schedule; records per-iteration losses and plans.

    ``gpu``: one GPU per rank, NCCL training groups, the bf16 kernels; every rank
    finishes its GPU work before the kill point (nothing is in flight when a rank dies),
    and after each recovery the rank checks its installed state against the checkpoint
    the recovery resumed from (principle A1) and records the mismatches."""
    _setup(env)
    import torch

    from harness import write_result
    from resihp.config import TrainConfig
    from resihp.control import ConsistentStop, ControlPlane
    from resihp.plan import build_plan
    from resihp.recovery import initial_run
    from resihp.train import fail_stop

    config = TrainConfig(**config_dict)
    schedule = {int(k): v for k, v in failures.items()}
    os.chdir(out_dir)
    device, backend = _device(gpu)
    cp = ControlPlane.initialize(training_backend=backend, memory_budget=config.memory_budget_bytes, device=device)
    plan = build_plan(config, step=0, version=0, memory_budget=config.memory_budget_bytes,
                      vocab_size=config.vocab_size, sequence_length=config.seq_len)
    groups = cp.build_training_groups(plan)
    cp.attach_run(initial_run(plan, rank=rank, groups=groups, device=device),
                  checkpoint_path=Path(out_dir, "checkpoint.pt"), device=device)
    record = {"rank": rank, "losses": {}, "plans": [plan.digest], "stopped": None, "recoveries": []}
    failed = ()
    try:
        it = 0
        while it < config.iterations:
            it += 1
            loss = cp.training_step()
            if loss is not None:
                record["losses"][str(it)] = loss
            if it % config.checkpoint_every == 0:
                cp.commit_checkpoint(plan, cursor=it)
            cp.quiesce()
            write_result(out_dir, rank, record)
            fail_stop(schedule, rank, it, before=cp.flush_checkpoint)
            lost = cp.observe()
            if lost:
                import shutil

                plan, failed = cp.safe_point(config, plan, failed, lost, next_step=it)
                # the lowest survivor keeps the checkpoint this failure resumed from
                ck = Path(out_dir, "checkpoint.pt")
                if rank == min(cp.members) and ck.exists():
                    shutil.copy(ck, Path(out_dir, f"anchor_{it}.pt"))
                entry = {"after": it, "lost": list(lost), "phases": cp.last_recovery, "resumed_from": cp.resume_cursor}
                if gpu and ck.exists():
                    from resihp.checkpoint import load_anchor
                    from resihp.recovery import checkpoint_mismatches

                    anchor, completed = load_anchor(ck)
                    entry["a1_completed"] = completed
                    entry["a1_mismatches"] = ([] if cp.training_run is None else
                                              checkpoint_mismatches(cp.training_run, plan=plan, rank=rank, anchor=anchor))
                if gpu and cp.training_run is not None:
                    red = cp.training_run.runtime.reducer
                    entry["reduction"] = ("none" if red is None else "p2p-hetero" if red.hetero is not None
                                          else "fused-dp" if red.fused_dp is not None else "nccl")
                record["plans"].append(plan.digest)
                record["recoveries"].append(entry)
                it = cp.resume_cursor
    except ConsistentStop as stop:
        record["stopped"] = stop.reason.code
        write_result(out_dir, rank, record)
        cp.shutdown()
        return
    write_result(out_dir, rank, record)
    cp.shutdown()


def rerun_entry(rank, env, config_dict, failed, after, anchor_path, out_dir, gpu=False):
    """Uninterrupted re-run of the post-failure plan from the anchor the failure resumed from."""
    _setup(env)
    from harness import write_result
    from resihp.checkpoint import load_anchor
    from resihp.config import TrainConfig
    from resihp.control import ControlPlane
    from resihp.plan import build_plan
    from resihp.recovery import run_from_anchor

    config = TrainConfig(**config_dict)
    survivors = [r for r in range(config.world_size) if r not in failed]
    plan_rank = survivors[rank]
    v0 = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    plan = build_plan(config, step=after, version=1, failed_ranks=failed, previous=v0,
                      vocab_size=config.vocab_size, sequence_length=config.seq_len)
    import torch.distributed as dist

    from resihp import membership

    store = membership.connect(os.environ[membership.HOST_ENV], os.environ[membership.PORT_ENV])
    device, backend = _device(gpu)
    cp = ControlPlane(plan_rank, survivors, store, backend, device=device)
    cp.form_world(survivors, epoch=0)
    groups = cp.build_training_groups(plan)
    anchor, completed = load_anchor(anchor_path)
    run = run_from_anchor(plan, rank=plan_rank, anchor=anchor, completed=completed, groups=groups, device=device)
    losses = {}
    for it in range(completed + 1, config.iterations + 1):
        loss = run.step() if run is not None else None
        if loss is not None:
            losses[str(it)] = loss
    write_result(out_dir, rank, {"rank": plan_rank, "losses": losses, "plan": plan.digest})
    cp.shutdown()


def a2_entry(rank, env, config_dict, anchor_path, start, out_dir):
    """Resume a TP run from an anchor, take one step, compare shards to the A2 oracle."""
    _setup(env)
    from harness import write_result
    from resihp import verify
    from resihp.checkpoint import load_anchor
    from resihp.config import TrainConfig
    from resihp.control import ControlPlane
    from resihp.plan import build_plan
    from resihp.recovery import run_from_anchor

    config = TrainConfig(**config_dict)
    cp = ControlPlane.initialize(training_backend="gloo")
    plan = build_plan(config, step=start, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    groups = cp.build_training_groups(plan)
    anchor, completed = load_anchor(anchor_path)
    run = run_from_anchor(plan, rank=rank, anchor=anchor, completed=completed, groups=groups)
    a1 = verify.matches_checkpoint(run, plan=plan, rank=rank, checkpoint_path=anchor_path)
    run.step()
    record = verify.steps_from_anchor(config, anchor, start=completed, count=1)[0]
    cmp = verify.compare_shards(run.stage, record, lr=config.lr)
    write_result(out_dir, rank, {"rank": rank, "a1": a1, "cmp": cmp})
    cp.shutdown()


def planned_entry(rank, env, config_dict, failed, steps, out_dir):
    """Train the plan a failure sequence leads to, from the seeded initialisation.

    ``rank`` indexes the survivors; no recovery happens -- this isolates the numerics of
    a post-failure layout (heterogeneous TP boundaries, migrated layers, replicas with
    different layouts reduced through the logical path).
    """
    _setup(env)
    from harness import write_result
    from resihp import membership
    from resihp.config import TrainConfig
    from resihp.control import ControlPlane
    from resihp.plan import build_plan
    from resihp.recovery import initial_run

    config = TrainConfig(**config_dict)
    survivors = [r for r in range(config.world_size) if r not in failed]
    plan_rank = survivors[rank]
    plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    seen = []
    for i, r in enumerate(failed):
        seen.append(r)
        plan = build_plan(config, step=i + 1, version=plan.version + 1, failed_ranks=tuple(seen), previous=plan,
                          vocab_size=config.vocab_size, sequence_length=config.seq_len)
    store = membership.connect(os.environ[membership.HOST_ENV], os.environ[membership.PORT_ENV])
    cp = ControlPlane(plan_rank, survivors, store, "gloo")
    cp.form_world(survivors, epoch=0)
    groups = cp.build_training_groups(plan)
    run = initial_run(plan, rank=plan_rank, groups=groups)
    losses = [run.step() if run is not None else None for _ in range(steps)]
    from resihp.recovery import stage_of

    stage = stage_of(plan, plan_rank)
    result = {"rank": plan_rank, "losses": losses, "replica": None if stage is None else stage.replica_id}
    if run is not None:
        result.update(shards={n: t.detach().tolist() for n, (t, _d) in run.stage.local_shards().items()},
                      tp_rank=run.stage.tp_rank, tp_size=run.stage.tp_size,
                      dims={n: d for n, (_t, d) in run.stage.local_shards().items()})
    write_result(out_dir, rank, result)
    cp.shutdown()


def e2e_entry(rank, env, config_dict, failures, out_dir):
    """The worker loop with a per-iteration account for the end-to-end invariants.

    Every iteration records the data cursor consumed, the plan version, the names this
    rank owns and (on a stage's first TP rank) the (micro-batch, stage, replica) pairs it
    executed; every recovery records whether the state equals the checkpoint before the
    first resumed step (principle A1). The file is rewritten after each iteration, so a
    killed rank leaves exactly the iterations it lived through.
    """
    _setup(env)
    import torch.distributed as dist

    from harness import write_result
    from resihp import verify
    from resihp.config import TrainConfig
    from resihp.control import ConsistentStop, ControlPlane
    from resihp.plan import build_plan
    from resihp.recovery import initial_run, stage_of
    from resihp.train import fail_stop

    config = TrainConfig(**config_dict)
    schedule = {int(k): v for k, v in failures.items()}
    os.chdir(out_dir)
    ck = Path(out_dir, "checkpoint.pt")
    cp = ControlPlane.initialize(training_backend="gloo")
    plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    groups = cp.build_training_groups(plan)
    cp.attach_run(initial_run(plan, rank=rank, groups=groups), checkpoint_path=ck)
    record = {"rank": rank, "iterations": [], "plans": [plan.digest], "recoveries": [], "stopped": None,
              "groups": [len(dist.distributed_c10d._world.pg_map)]}
    failed = ()
    try:
        it = 0
        while it < config.iterations:
            it += 1
            run = cp.training_run
            entry = {"iteration": it, "plan_version": plan.version, "trained": run is not None}
            if run is not None:
                stage = stage_of(plan, rank)
                entry.update(cursor=run.cursor, owned=sorted(run.stage.local_shards()), replica=stage.replica_id,
                             stage=stage.stage_id, leader=stage.tp_members[0] == rank)
            loss = cp.training_step()
            if run is not None:
                entry["loss"] = loss
                if entry["leader"]:
                    entry["executed"] = [int(x[1:]) for x in run.runtime.schedule if x.startswith("F")]
            record["iterations"].append(entry)
            cp.commit_checkpoint(plan, cursor=it)
            write_result(out_dir, rank, record)
            fail_stop(schedule, rank, it, before=cp.flush_checkpoint)
            lost = cp.observe()
            if lost:
                import shutil

                plan, failed = cp.safe_point(config, plan, failed, lost, next_step=it)
                if rank == min(cp.members):
                    shutil.copy(ck, Path(out_dir, f"anchor_{it}.pt"))
                a1 = None
                if cp.training_run is not None:
                    a1 = verify.matches_checkpoint(cp.training_run, plan=plan, rank=rank, checkpoint_path=ck)
                record["plans"].append(plan.digest)
                record["groups"].append(len(dist.distributed_c10d._world.pg_map))
                record["recoveries"].append({"after": it, "lost": list(lost), "a1": a1,
                                             "resumed_from": cp.resume_cursor, "version": plan.version})
                it = cp.resume_cursor
    except ConsistentStop as stop:
        record["stopped"] = stop.reason.code
    cp.shutdown()
    record["initialized"] = dist.is_initialized()
    write_result(out_dir, rank, record)


def churn_entry(rank, env, config_dict, churn_after, out_dir):
    """Train; optionally tear every group down after ``churn_after`` iterations and rebuild
    the world, the groups and the run from its own live state under the same plan."""
    _setup(env)
    from harness import write_result
    from resihp.config import TrainConfig
    from resihp.control import ControlPlane
    from resihp.plan import build_plan
    from resihp.recovery import initial_run, recover

    config = TrainConfig(**config_dict)
    os.chdir(out_dir)
    cp = ControlPlane.initialize(training_backend="gloo")
    plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    groups = cp.build_training_groups(plan)
    ck = Path(out_dir, "checkpoint.pt")
    cp.attach_run(initial_run(plan, rank=rank, groups=groups), checkpoint_path=ck)
    losses = []
    for it in range(1, config.iterations + 1):
        losses.append(cp.training_step())
        cp.commit_checkpoint(plan, cursor=it)
        cp.flush_checkpoint()
        if it == churn_after:
            cp.dissolve_world()
            cp.form_world(cp.members, epoch=cp.epoch + 1)
            groups = cp.build_training_groups(plan)
            cp.training_run, _digest, _cursor = recover(cp.training_run, plan=plan, previous=plan, rank=rank,
                                                        cursor=it, checkpoint_path=ck, groups=groups)
    write_result(out_dir, rank, {"rank": rank, "losses": losses})
    cp.shutdown()
