"""The run's entry point: spawn one worker per rank, host the store, outlive the dead.

``python3 -m resihp.launch --config train.json --failures failures.json [--timeout S] [--resume CK]``
(reference ``resihp/launch.py:44-110``). ``torchrun`` cannot host a fail-stop run: its
agent treats a worker killed by a signal as a job failure and restarts the survivors,
whereas recovery here is an in-place reconfiguration of the survivors. The launcher
hosts the ``TCPStore`` (so no rank's death takes the rendezvous with it), spawns
``world_size = tp * pp * dp`` workers with ``RANK``/``LOCAL_RANK``/``WORLD_SIZE`` set,
and exits 0 only when exactly the scheduled ranks died of ``SIGKILL`` and every other
rank exited cleanly.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
from pathlib import Path

from .config import load_config
from .membership import Supervisor

DEFAULT_TIMEOUT = 900.0
KILLED = -9


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="resihp fail-stop launcher")
    p.add_argument("--config", required=True, type=Path)
    p.add_argument("--failures", required=True, type=Path)
    p.add_argument("--timeout", type=float, default=DEFAULT_TIMEOUT)
    p.add_argument("--resume", type=Path, default=None,
                   help="restart a stopped job from this checkpoint (the layout may differ)")
    return p.parse_args(argv)


def _restart_point(resume: Path | None) -> int:
    """Iterations the checkpoint ``resume`` has completed (0 for a fresh job)."""
    if resume is None:
        return 0
    from .checkpoint import completed_steps

    return completed_steps(resume)


def launch(config_path: Path, failures_path: Path, *, timeout: float = DEFAULT_TIMEOUT, resume: Path | None = None):
    """Run the job; ``(exit codes by rank, ranks the schedule kills)``. With ``resume``
    the job restarts from that checkpoint and only the failures after it are scheduled."""
    loaded = load_config(config_path, failures_path)
    world = loaded.train.world_size
    start = _restart_point(resume)
    scheduled = sorted(e.failed_rank for e in loaded.failures if e.after_iteration > start)
    sup = Supervisor(range(world))
    for rank in range(world):
        env = {**os.environ, **sup.env(), "RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(world)}
        cmd = [sys.executable, "-m", "resihp.train", "--config", str(config_path), "--failures", str(failures_path)]
        if resume is not None:
            cmd += ["--resume", str(Path(resume).resolve())]
        sup.register(rank, subprocess.Popen(cmd, env=env))
    return sup.serve(timeout=timeout), scheduled


def main(argv=None) -> int:
    args = parse_args(argv)
    codes, scheduled = launch(args.config, args.failures, timeout=args.timeout, resume=args.resume)
    killed = sorted(r for r, c in codes.items() if c == KILLED)
    survivors = {r: c for r, c in codes.items() if r not in scheduled}
    ok = killed == scheduled and set(survivors.values()) <= {0}
    print(json.dumps({"launch": {"world_size": len(codes), "killed_ranks": killed, "scheduled_kills": scheduled,
                                 "exit_codes": {str(r): codes[r] for r in sorted(codes)}}}), flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
