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


class Supervisor:
    """Store host, process table and the run's only liveness authority (not a rank)."""

    def __init__(self, ranks, *, host: str = "127.0.0.1", port: int | None = None):
        from torch.distributed import TCPStore

        self.host = host
        self.port = free_port() if port is None else int(port)
        self.ranks = tuple(sorted(ranks))
        self.store = TCPStore(self.host, self.port, is_master=True, wait_for_workers=False, timeout=DEFAULT_TIMEOUT)
        self._children: dict[int, object] = {}
        self.exit_codes: dict[int, int] = {}
        self.published: list[tuple[int, tuple[int, ...], float]] = []

    def env(self) -> dict[str, str]:
        return {HOST_ENV: self.host, PORT_ENV: str(self.port)}

    def register(self, rank: int, child) -> None:
        self._children[int(rank)] = child

    @property
    def alive(self) -> tuple[int, ...]:
        return tuple(r for r in self.ranks if r not in self.exit_codes)

    def _reap(self) -> None:
        for rank in self.alive:
            child = self._children[rank]
            code = child.poll() if hasattr(child, "poll") else child.exitcode
            if code is not None:
                self.exit_codes[rank] = int(code)

    def serve(self, *, timeout: float) -> dict[int, int]:
        """Publish one membership per boundary until every worker has exited."""
        deadline = time.monotonic() + timeout
        iteration = 1
        while True:
            self._reap()
            if not self.alive:
                return dict(self.exit_codes)
            arrived = self.store.add(ARRIVALS.format(iteration=iteration), 0)
            if arrived >= len(self.alive):
                members = list(self.alive)
                self.store.set(MEMBERS.format(iteration=iteration), json.dumps(members))
                self.published.append((iteration, tuple(members), time.time()))
                iteration += 1
                continue
            if time.monotonic() > deadline:
                self.kill_all()
                raise TimeoutError(
                    f"boundary {iteration}: {arrived} of {len(self.alive)} live ranks arrived within "
                    f"{timeout}s (alive={list(self.alive)})"
                )
            time.sleep(POLL_SECONDS)

    def kill_all(self) -> None:
        """Last resort for a stuck run (not part of the failure model)."""
        import os
        import signal

        for rank in self.alive:
            try:
                os.kill(self._children[rank].pid, signal.SIGKILL)
            except (ProcessLookupError, PermissionError):
                pass
