"""Store-backed membership: liveness from the launcher's process table.

The launcher (:class:`Supervisor`) hosts the run's ``TCPStore`` and owns the worker
processes; a rank is gone exactly when the operating system reports its exit. Every
iteration boundary is a rendezvous on that store: each live rank adds itself to the
boundary's arrival counter and waits for the supervisor to publish the boundary's
membership, which it does once every process still running has arrived. A rank killed
at a safe point never arrives, so the survivors read a membership that already
excludes it before they issue another collective. Protocol and keys follow the
reference (``resihp/membership.py:31-174``): ``boundary/<i>/arrivals``,
``boundary/<i>/members`` and the per-epoch world prefix ``world/<epoch>/``.
No heartbeats and no timeouts are part of the failure model; the timeouts here only
turn a stuck run into an error.
"""

from __future__ import annotations

import json
import socket
import time
from datetime import timedelta

ARRIVALS = "boundary/{iteration}/arrivals"
MEMBERS = "boundary/{iteration}/members"
PG_PREFIX = "world/{epoch}/"
HOST_ENV = "RESIHP_STORE_HOST"
PORT_ENV = "RESIHP_STORE_PORT"
DEFAULT_TIMEOUT = timedelta(seconds=300)
POLL_SECONDS = 0.02


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def connect(host: str, port, timeout: timedelta = DEFAULT_TIMEOUT):
    from torch.distributed import TCPStore

    return TCPStore(host, int(port), is_master=False, timeout=timeout)


def boundary(store, iteration: int, *, timeout: timedelta = DEFAULT_TIMEOUT) -> tuple[int, ...]:
    """Arrive at boundary ``iteration`` and return the membership the supervisor published."""
    store.add(ARRIVALS.format(iteration=iteration), 1)
    key = MEMBERS.format(iteration=iteration)
    store.wait([key], timeout)
    return tuple(json.loads(store.get(key)))


def _exit_status(child) -> int | None:
    """Exit status of a spawned worker, or None while it runs: ``subprocess.Popen``
    children answer ``poll()``, ``multiprocessing.Process`` children expose
    ``exitcode``; both report a signal death as the negative signal number."""
    poll = getattr(child, "poll", None)
    status = poll() if callable(poll) else child.exitcode
    return None if status is None else int(status)


class Supervisor:
    """Host of the run's store and its only liveness authority (not a rank).

    It keeps a process table of the workers it was handed and, in :meth:`serve`,
    alternates two duties until every worker has exited: fold newly exited workers into
    ``exit_codes`` (the operating system's verdict, never a guess), and publish every
    boundary whose arrival counter already covers all workers still running. The
    membership it publishes for a boundary is exactly that running set, so a worker
    killed before it arrived is absent from it. ``published`` records
    ``(boundary, members, wall time)`` for every publication.
    """

    def __init__(self, ranks, *, host: str = "127.0.0.1", port: int | None = None):
        from torch.distributed import TCPStore

        self.host = host
        self.port = int(port) if port is not None else free_port()
        self.ranks = tuple(sorted(ranks))
        self.store = TCPStore(self.host, self.port, is_master=True, wait_for_workers=False, timeout=DEFAULT_TIMEOUT)
        self.exit_codes: dict[int, int] = {}
        self.published: list[tuple[int, tuple[int, ...], float]] = []
        self._workers: dict[int, object] = {}
        self._next_boundary = 1

    def env(self) -> dict[str, str]:
        """Store address for a worker's environment."""
        return {HOST_ENV: self.host, PORT_ENV: str(self.port)}

    def register(self, rank: int, child) -> None:
        self._workers[int(rank)] = child

    @property
    def alive(self) -> tuple[int, ...]:
        """Ranks whose process has not exited, ascending."""
        return tuple(sorted(set(self.ranks).difference(self.exit_codes)))

    def refresh(self) -> None:
        """Record the exit status of every worker that has ended since the last look."""
        ended = {rank: _exit_status(self._workers[rank]) for rank in self.alive}
        self.exit_codes.update({rank: code for rank, code in ended.items() if code is not None})

    def publish_ready(self) -> int:
        """Publish each pending boundary that every running worker has reached; returns
        how many were published."""
        count = 0
        running = self.alive
        while running and self.store.add(ARRIVALS.format(iteration=self._next_boundary), 0) >= len(running):
            self.store.set(MEMBERS.format(iteration=self._next_boundary), json.dumps(list(running)))
            self.published.append((self._next_boundary, running, time.time()))
            self._next_boundary += 1
            count += 1
        return count

    def serve(self, *, timeout: float) -> dict[int, int]:
        """Run the boundary service until every worker has exited and return the exit
        codes. ``timeout`` bounds the whole run: it only catches a stuck worker (no
        timeout is part of the failure model), so on expiry every worker is killed and
        :class:`TimeoutError` names the boundary that never completed."""
        give_up = time.monotonic() + timeout
        while True:
            self.refresh()
            if self.publish_ready():
                continue  # look at the process table again before the next boundary
            if not self.alive:
                return dict(self.exit_codes)
            if time.monotonic() >= give_up:
                waiting = self.store.add(ARRIVALS.format(iteration=self._next_boundary), 0)
                self.kill_all()
                raise TimeoutError(
                    f"run exceeded {timeout}s at boundary {self._next_boundary}: only {waiting} of the "
                    f"running ranks {list(self.alive)} arrived")
            time.sleep(POLL_SECONDS)

    def kill_all(self) -> None:
        """Send SIGKILL to every worker still running (the stuck-run last resort)."""
        import os
        import signal

        for rank in self.alive:
            pid = getattr(self._workers[rank], "pid", None)
            if pid is None:
                continue
            try:
                os.kill(pid, signal.SIGKILL)
            except (ProcessLookupError, PermissionError):
                continue
