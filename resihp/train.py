"""One rank's training process: the fail-stop control loop, or a config echo.

``python -m resihp.train --config train.json --failures failures.json`` is what the
launcher spawns per rank (reference ``resihp/train.py:75-188``). Without ``RANK`` in
the environment it only echoes the two files as JSON.

Each iteration: train (1F1B over the plan), commit the logical checkpoint (every
``checkpoint_every`` iterations; every iteration by default, as the reference), then
-- if the schedule names this rank -- ``SIGKILL`` itself, then rendezvous at the
boundary; a boundary that comes back short triggers exactly one safe point. The JSON
lines on stdout are the reference's ``{"acceptance": ...}`` / ``{"stopped": ...}``
plus ``{"step": ...}`` per trained iteration on a last-stage rank and
``{"recovery": ...}`` per fail-stop.
"""

from __future__ import annotations

import argparse
import json
import os
import time
from pathlib import Path

from .config import TrainConfig, load_config

CHECKPOINT_PATH = Path(os.environ.get("RESIHP_CHECKPOINT", "checkpoint.pt"))
#: Token-stream shape of a config that does not set ``vocab_size`` / ``seq_len`` (the
#: reference's run constants, ``resihp/train.py:37-38``); a config's fields override them.
VOCAB_SIZE = TrainConfig.__dataclass_fields__["vocab_size"].default
SEQUENCE_LENGTH = TrainConfig.__dataclass_fields__["seq_len"].default


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="resihp training worker")
    p.add_argument("--config", required=True, type=Path)
    p.add_argument("--failures", required=True, type=Path)
    p.add_argument("--resume", type=Path, default=None,
                   help="restart a stopped job from this checkpoint (any TP/PP/DP layout)")
    return p.parse_args(argv)


def select_device():
    """This rank's GPU (``LOCAL_RANK``), or the CPU where there is none.

    One rank per GPU is a hard rule, not a default: the fused kernels of ranks that wait
    on one another must run concurrently, which two launches sharing one GPU do not
    guarantee. A job with more ranks than visible GPUs is refused.
    """
    import torch

    if not torch.cuda.is_available():
        return torch.device("cpu")
    local = int(os.environ.get("LOCAL_RANK", 0))
    if local >= torch.cuda.device_count():
        raise RuntimeError(f"rank with LOCAL_RANK={local} has no GPU of its own: {torch.cuda.device_count()} visible; "
                           "run one rank per GPU")
    torch.cuda.set_device(local)
    return torch.device("cuda", torch.cuda.current_device())


def fail_stop(schedule, rank: int, iteration: int, *, before=None) -> None:
    """``SIGKILL`` this process if the schedule fails ``rank`` after ``iteration``.

    ``schedule`` maps an iteration to the rank (or a collection of ranks, for tests of
    simultaneous failures; failure files name one rank per event) that fails after it.
    ``before`` runs first (the worker passes its checkpoint flush, so a scheduled
    fail-stop happens after its iteration's commit is on disk).
    """
    import signal

    victims = schedule.get(iteration)
    if victims == rank or (isinstance(victims, (list, tuple, set, frozenset)) and rank in victims):
        if before is not None:
            before()
        os.kill(os.getpid(), signal.SIGKILL)


def _emit(obj) -> None:
    """One JSON line in a single write, so lines of concurrent ranks never interleave."""
    import sys

    sys.stdout.write(json.dumps(obj, ensure_ascii=False) + "\n")
    sys.stdout.flush()


def _resumed_run(path: Path, config, plan, *, rank, groups, device):
    """``(run, completed steps)`` rebuilt from a checkpoint under ``plan``.

    The checkpoint is topology-free, so the restarted job may run another layout; the
    installed shards are checked against the checkpoint (principle A1) before training.
    """
    from .checkpoint import CheckpointError, load_checkpoint
    from .recovery import checkpoint_mismatches, run_from_anchor

    anchor, completed, _version = load_checkpoint(path, config)  # validated; restores the RNG
    if completed >= config.iterations:
        raise CheckpointError(f"checkpoint {path} already holds {completed} of {config.iterations} iterations")
    run = run_from_anchor(plan, rank=rank, anchor=anchor, completed=completed, groups=groups, device=device)
    problems = [] if run is None else checkpoint_mismatches(run, plan=plan, rank=rank, anchor=anchor)
    if problems:
        raise CheckpointError(f"rank {rank} state differs from {path} after the restart: {problems[:5]}")
    return run, completed


def _adopt_checkpoint(resume: Path, checkpoint_path: Path, control) -> None:
    """Make the restart point this job's checkpoint too, so a failure before the job's own
    first commit rolls back to it. The lowest rank links (or copies) the file into place
    atomically; the others wait for it."""
    import shutil

    import torch.distributed as dist

    src, dst = Path(resume).resolve(), Path(checkpoint_path).resolve()
    if src != dst and control.rank == min(control.members):
        tmp = dst.with_name(dst.name + ".adopt")
        if tmp.exists():
            tmp.unlink()
        try:
            os.link(src, tmp)
        except OSError:
            shutil.copyfile(src, tmp)
        os.replace(tmp, dst)
    dist.barrier(group=control.world_group)


def run_distributed(loaded, *, checkpoint_path: Path = CHECKPOINT_PATH, resume: Path | None = None):
    """One rank's whole job. ``resume`` restarts it from a checkpoint: training continues
    after the checkpoint's completed iterations, and failure events at or before them are
    in the past."""
    import torch

    from .checkpoint import completed_steps
    from .control import ConsistentStop, ControlPlane
    from .plan import build_plan
    from .recovery import initial_run

    config = loaded.train
    schedule = {e.after_iteration: e.failed_rank for e in loaded.failures}
    device = select_device()
    control = ControlPlane.initialize(memory_budget=config.memory_budget_bytes, device=device)
    start = 0 if resume is None else completed_steps(resume)
    plan = build_plan(
        config, step=start, version=0, memory_budget=config.memory_budget_bytes,
        vocab_size=config.vocab_size, sequence_length=config.seq_len,
    )
    groups = control.build_training_groups(plan)
    if resume is None:
        run = initial_run(plan, rank=control.rank, groups=groups, device=device)
    else:
        run, start = _resumed_run(resume, config, plan, rank=control.rank, groups=groups, device=device)
        _adopt_checkpoint(resume, checkpoint_path, control)
        _emit({"resume": {"rank": control.rank, "checkpoint": str(resume), "completed_steps": start}})
    control.attach_run(run, checkpoint_path=checkpoint_path, device=device)
    failed: tuple[int, ...] = ()
    pending_recovery = None
    trained: list[int] = []
    versions = [plan.version]
    digests = [plan.digest]
    tokens_per_step = config.batch_size * config.seq_len
    try:
        iteration = start
        while iteration < config.iterations:
            iteration += 1
            if control.training_run is not None:
                trained.append(iteration)
            t0 = time.perf_counter()
            events = None
            if device.type == "cuda":
                events = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                events[0].record()
            loss = control.training_step()
            if events is not None:
                events[1].record()
                torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            if loss is not None:
                _emit({"step": iteration, "rank": control.rank, "loss": loss, "plan_version": plan.version,
                       "step_s": dt, "tokens_per_s": tokens_per_step / dt if dt > 0 else None,
                       "device_ms": None if events is None else events[0].elapsed_time(events[1])})
            if pending_recovery is not None:
                # failure -> end of the first resumed step, as seen by this rank
                pending_recovery["seconds"] = time.perf_counter() - pending_recovery.pop("t_fail")
                pending_recovery["first_step_s"] = dt
                _emit({"recovery": pending_recovery})
                pending_recovery = None
            if iteration % config.checkpoint_every == 0:
                control.commit_checkpoint(plan, cursor=iteration)
            control.quiesce()  # the iteration, its commit and all their GPU work are complete
            fail_stop(schedule, control.rank, iteration, before=control.flush_checkpoint)
            t_fail = time.perf_counter()
            lost = control.observe()
            if lost:
                plan, failed = control.safe_point(config, plan, failed, lost, next_step=iteration)
                versions.append(plan.version)
                digests.append(plan.digest)
                pending_recovery = {"rank": control.rank, "event": len(versions) - 1, "lost": list(lost),
                                    "after_iteration": iteration, "plan_version": plan.version,
                                    "resumed_from": control.resume_cursor,
                                    "safe_point_s": time.perf_counter() - t_fail,
                                    "phases": control.last_recovery, "t_fail": t_fail}
                # a rollback to an older checkpoint re-runs the iterations after it
                iteration = control.resume_cursor
        if pending_recovery is not None:
            pending_recovery.pop("t_fail")
            pending_recovery["seconds"] = pending_recovery["safe_point_s"]
            _emit({"recovery": pending_recovery})
    except ConsistentStop as stop:
        _emit({"stopped": stop.reason.code, "reason": stop.reason.message})
        control.shutdown()
        return None
    _emit({"acceptance": {
        "rank": control.rank, "device": device.type, "training_backend": control.training_backend,
        "trained_iterations": trained, "plan_versions": versions, "plan_digests": digests,
        "failed_ranks": list(failed), "world_members": list(control.members),
    }})
    control.shutdown()
    return plan


def main(argv=None):
    args = parse_args(argv)
    if "RANK" in os.environ:
        run_distributed(load_config(args.config, args.failures), resume=args.resume)
        return
    config = json.loads(args.config.read_text(encoding="utf-8"))
    failures = json.loads(args.failures.read_text(encoding="utf-8"))
    print(json.dumps({"config": config, "failures": failures}, ensure_ascii=False, sort_keys=True))


if __name__ == "__main__":
    main()
