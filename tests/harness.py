"""Multi-process fail-stop harness: one process per plan rank, SIGKILL means gone.

The same machinery the launcher uses: a :class:`resihp.membership.Supervisor` hosts the
store and is the process table; each rank is a ``spawn`` child that installs its
``RANK``/``WORLD_SIZE``/store environment before touching torch. A rank that kills itself
simply stops being expected at the next boundary.
"""

import json
import os
from pathlib import Path

from resihp.membership import Supervisor

JOIN_TIMEOUT = 600.0
KILLED = -9


def run_ranks(entry, world_size, *extra, timeout=JOIN_TIMEOUT):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    sup = Supervisor(range(world_size))
    shared = {**sup.env(), "WORLD_SIZE": str(world_size)}
    for rank in range(world_size):
        env = {**shared, "RANK": str(rank), "LOCAL_RANK": str(rank)}
        child = ctx.Process(target=entry, args=(rank, env, *extra))
        child.start()
        sup.register(rank, child)
    return sup.serve(timeout=timeout)


def read_results(directory, ranks):
    return {r: json.loads(Path(directory, f"result_{r}.json").read_text()) for r in ranks}


def write_result(directory, rank, obj):
    tmp = Path(directory, f"result_{rank}.json.tmp")
    tmp.write_text(json.dumps(obj))
    os.replace(tmp, Path(directory, f"result_{rank}.json"))


def assert_killed(exit_codes, killed, label=""):
    expected = {r: (KILLED if r in set(killed) else 0) for r in sorted(exit_codes)}
    assert exit_codes == expected, (label, exit_codes, expected)
