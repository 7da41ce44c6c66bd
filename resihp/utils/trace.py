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


# kernel name pattern -> category, first match wins (names as the torch profiler reports
# them, demangled or mangled; the GEMM's template arguments say which linear-layer
# product it is: <BN, A MN-major, B MN-major, epilogue> for the single-CTA kernel,
# <A MN-major, B MN-major, epilogue, stages> for the CTA-pair kernel)
_CATEGORIES = (
    (r"fused_gemm_kernel", "fused TP collective GEMM"),
    (r"gemm_kernel<\d+, false, false|gemm_kernelILi\d+ELb0ELb0E"
     r"|gemm_pair_kernel<false, false|gemm_pair_kernelILb0ELb0E", "GEMM forward"),
    (r"gemm_kernel<\d+, false, true|gemm_kernelILi\d+ELb0ELb1E"
     r"|gemm_pair_kernel<false, true|gemm_pair_kernelILb0ELb1E", "GEMM dgrad"),
    (r"gemm_kernel<\d+, true, true|gemm_kernelILi\d+ELb1ELb1E"
     r"|gemm_pair_kernel<true, true|gemm_pair_kernelILb1ELb1E", "GEMM wgrad"),
    (r"gemm_(pair_)?kernel", "GEMM other"),
    (r"attn_fwd_kernel", "attention forward"),
    (r"attn_bwd|attn_delta", "attention backward"),
    (r"rmsnorm|column_sum", "RMSNorm"),
    (r"rope(_vec)?_kernel|swiglu|embedding_(fwd|bwd|sort)_kernel", "RoPE / SwiGLU / embedding"),
    (r"xent_", "cross-entropy"),
    (r"dp_adamw(_push)?_kernel", "fused DP all-reduce + AdamW"),
    (r"adamw(_vec)?_kernel", "AdamW"),
    (r"reshard_gather", "state move"),
    (r"(?i)nccl", "NCCL"),
    (r"(?i)memcpy|memset", "copies"),
)


def categorize(rows) -> dict:
    """Device time per kernel category from ``[{"name", "calls", "device_us"}]`` rows:
    ``{category: {"device_us", "calls", "share"}}``, largest first. What matches no
    pattern (torch's own elementwise kernels, fills) is ``"other"``."""
    import re

    totals: dict[str, list] = {}
    for row in rows:
        name = row["name"]
        cat = next((c for pattern, c in _CATEGORIES if re.search(pattern, name)), "other")
        entry = totals.setdefault(cat, [0.0, 0])
        entry[0] += float(row["device_us"])
        entry[1] += int(row["calls"])
    whole = sum(v[0] for v in totals.values()) or 1.0
    ordered = sorted(totals.items(), key=lambda kv: -kv[1][0])
    return {c: {"device_us": round(us, 1), "calls": n, "share": round(us / whole, 4)} for c, (us, n) in ordered}
