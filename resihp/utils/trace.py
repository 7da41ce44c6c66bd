"""NVTX ranges for profiler timelines, off unless ``RESIHP_NVTX=1``.

The 1F1B runtime marks every micro-batch's forward ``F<i>`` and backward ``B<i>``, each
pipeline exchange ``p2p`` and the gradient-reduction + optimizer step ``W`` (the same
labels as :attr:`resihp.parallel.pp.PipelineRuntime.schedule`); the control plane marks
the checkpoint commit and every safe-point phase. Disabled, :func:`nvtx_range` is a
no-op context manager, so the hot path pays nothing. (The reference has no tracing; its
only execution record is the schedule list of ``resihp/parallel/pp.py:127,369``.)
"""

from __future__ import annotations

import contextlib
import os

ENABLED = os.environ.get("RESIHP_NVTX", "0") == "1"


def _available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover - torch always importable here
        return False


_ON = ENABLED and _available()


@contextlib.contextmanager
def _range(name: str):
    import torch

    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def nvtx_range(name: str):
    """A context manager that brackets its body with an NVTX range when tracing is on."""
    return _range(name) if _ON else contextlib.nullcontext()
