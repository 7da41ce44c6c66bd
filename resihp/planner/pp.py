"""Pipeline partitioning, the 1F1B schedule, and fail-stop layer repartition.

The 1F1B schedule is defined here, torch-free, because three parties must agree on it:
the runtime that executes it (:class:`resihp.parallel.pp.PipelineRuntime`), the memory
model that sizes its activation peak, and the DP gate that re-checks that peak on the
published layout. Same semantics as the reference (``resihp/planner/pp.py:16-245``):

* base partition: contiguous, the remainder going to the earlier stages;
* stage ``i`` of ``S`` runs ``w = min(S-1-i, M)`` warm-up forwards, then ``M-w``
  forward/backward pairs, then ``w`` cool-down backwards (``F^w (F B)^(M-w) B^w``);
* repartition after a TP-degree change: each surviving stage targets
  ``max(1, L_old * TP_new // TP_old)`` layers (0 for a dead stage); surplus layers go
  one at a time to the stage with the smallest layers/TP ratio, deficits are taken
  from the stage with the largest ratio that keeps at least one layer, ties to the
  lowest stage id. Ratios are compared by integer cross-multiplication, never floats.
"""

from __future__ import annotations

from dataclasses import dataclass

from ..validate import non_negative_int


def balanced_layers(num_layers: int, num_stages: int) -> tuple[tuple[int, ...], ...]:
    """Global layer ids per stage for the pristine partition."""
    if num_stages < 1 or num_layers < num_stages:
        raise ValueError("need at least one layer per stage")
    base, extra = divmod(num_layers, num_stages)
    out, start = [], 0
    for stage in range(num_stages):
        n = base + (stage < extra)
        out.append(tuple(range(start, start + n)))
        start += n
    return tuple(out)


def pipeline_phases(num_micro_batches: int, *, stage_index: int, num_stages: int) -> tuple[int, int]:
    """``(warmup, steady)`` counts of one stage's 1F1B schedule."""
    if num_stages < 1 or not 0 <= stage_index < num_stages:
        raise ValueError("stage_index must identify a stage of the pipeline")
    n = non_negative_int("num_micro_batches", num_micro_batches)
    warmup = min(num_stages - 1 - stage_index, n)
    return warmup, n - warmup


def pipeline_schedule(num_micro_batches: int, *, stage_index: int, num_stages: int) -> tuple[str, ...]:
    """The ``"F"``/``"B"`` issue order of one stage."""
    warmup, steady = pipeline_phases(num_micro_batches, stage_index=stage_index, num_stages=num_stages)
    return ("F",) * warmup + ("F", "B") * steady + ("B",) * warmup


def peak_in_flight(num_micro_batches: int, *, stage_index: int, num_stages: int) -> int:
    """High-water mark of live activations, replayed from :func:`pipeline_schedule`."""
    live = peak = 0
    for op in pipeline_schedule(num_micro_batches, stage_index=stage_index, num_stages=num_stages):
        live += 1 if op == "F" else -1
        peak = max(peak, live)
    return peak


@dataclass(frozen=True)
class PPInfeasibleReason:
    code: str
    message: str


class InfeasiblePP(ValueError):
    """No executable partition exists (stop code ``no_executable_pp``)."""

    def __init__(self, reason: PPInfeasibleReason):
        super().__init__(reason.message)
        self.reason = reason


@dataclass(frozen=True)
class PPPlan:
    stage_layers: tuple[int, ...]
    layer_ranges: tuple[tuple[int, int] | None, ...]
    migrations: tuple[tuple[int, int, int], ...]
    embedding_owner: int
    lm_head_owner: int


def _counts(name: str, values) -> tuple[int, ...]:
    out = tuple(non_negative_int(name, v) for v in values)
    if not out:
        raise ValueError(f"{name} must not be empty")
    return out


def owner_ranges(stage_layers: tuple[int, ...]) -> tuple[tuple[int, int] | None, ...]:
    """``(start, end)`` per stage laid out contiguously; ``None`` for an empty stage."""
    out, start = [], 0
    for n in stage_layers:
        out.append((start, start + n) if n else None)
        start += n
    return tuple(out)


def _owner_of(ranges, layer: int) -> int:
    for stage, bounds in enumerate(ranges):
        if bounds is not None and bounds[0] <= layer < bounds[1]:
            return stage
    raise AssertionError("layer ranges do not cover the model")


def _lighter(a: int, b: int, load: list[int], tp: tuple[int, ...]) -> bool:
    """Stage ``a`` carries fewer layers per TP rank than stage ``b`` (exact)."""
    return load[a] * tp[b] < load[b] * tp[a]


def _pick(stages: list[int], load: list[int], tp: tuple[int, ...], *, lightest: bool) -> int:
    """The lightest (or heaviest) stage; equal ratios resolve to the lowest stage id."""
    best = stages[0]
    for s in stages[1:]:
        better = _lighter(s, best, load, tp) if lightest else _lighter(best, s, load, tp)
        if better:
            best = s
    return best


def _balance(target: list[int], total: int, tp: tuple[int, ...]) -> None:
    active = [s for s, k in enumerate(tp) if k > 0]
    if not active:
        raise InfeasiblePP(PPInfeasibleReason("no_executable_pp", "all PP stages have zero TP capacity"))
    if len(active) > total:
        raise InfeasiblePP(PPInfeasibleReason("no_executable_pp", "active PP stages outnumber model layers"))
    gap = total - sum(target)
    while gap > 0:
        target[_pick(active, target, tp, lightest=True)] += 1
        gap -= 1
    while gap < 0:
        spare = [s for s in active if target[s] > 1]
        if not spare:
            raise InfeasiblePP(
                PPInfeasibleReason("no_executable_pp", "active PP stages cannot retain at least one layer each")
            )
        target[_pick(spare, target, tp, lightest=False)] -= 1
        gap += 1


def repartition_pp(old_stage_layers, old_tp_degrees, new_tp_degrees) -> PPPlan:
    """Redistribute contiguous layers after stages changed TP degree.

    An empty old stage is ``old_stage_layers == old_tp_degrees == 0``; a stage whose
    ranks all died has new degree 0 and ends with no layers.
    """
    old_layers = _counts("old_stage_layers", old_stage_layers)
    old_tp = _counts("old_tp_degrees", old_tp_degrees)
    new_tp = _counts("new_tp_degrees", new_tp_degrees)
    if not len(old_layers) == len(old_tp) == len(new_tp):
        raise ValueError("stage layer and TP degree sequences must have the same length")
    if any((n == 0) != (k == 0) for n, k in zip(old_layers, old_tp)):
        raise ValueError("empty old stages must have zero TP degree")
    total = sum(old_layers)
    if total == 0:
        raise ValueError("old_stage_layers must contain at least one layer")

    target = [
        0 if k_new == 0 or k_old == 0 else max(1, n * k_new // k_old)
        for n, k_old, k_new in zip(old_layers, old_tp, new_tp)
    ]
    _balance(target, total, new_tp)
    layers = tuple(target)
    if sum(layers) != total:
        raise AssertionError("PP layer count is not conserved")
    if any((k == 0 and n) or (k > 0 and n < 1) for n, k in zip(layers, new_tp)):
        raise AssertionError("PP stage executability invariant failed")

    before, after = owner_ranges(old_layers), owner_ranges(layers)
    moves = []
    for layer in range(total):
        src, dst = _owner_of(before, layer), _owner_of(after, layer)
        if src != dst:
            moves.append((layer, src, dst))
    live = [s for s, k in enumerate(new_tp) if k > 0]
    return PPPlan(layers, after, tuple(moves), live[0], live[-1])
