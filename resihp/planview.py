"""Preview the plans of a run without running it.

    python -m resihp.planview --config train.json [--failures failures.json]

Prints one JSON line per plan the schedule produces -- the initial plan, then one per
failure event -- or, where the planner has no answer, the consistent-stop line the job
would end with. Each plan line holds its version and step, the failed and active ranks,
the plan digest (the value every rank agrees on at the safe point), the stages
(replica, stage, TP members, layer range), the micro-batches each replica executes, the
state routes counted by reshard method, and the planner's memory estimate for the most
loaded rank against the budget. Pure planning: no process group, no torch; the same
functions the workers call (reference counterparts: ``resihp/plan.py:304-481`` and the
memory gate of ``resihp/memory.py:40-125``).
"""

from __future__ import annotations

import argparse
import json
from collections import Counter
from pathlib import Path

from .config import load_config, parse_train
from .memory import estimate_memory
from .plan import InfeasiblePlan, build_plan
from .planner.pp import peak_in_flight


def _stage_memory(plan, stage) -> int:
    """Planner estimate for one TP rank of ``stage`` (bytes)."""
    c = plan.config
    micro = sum(1 for p in plan.placements if p.replica_id == stage.replica_id and p.stage_id == stage.stage_id)
    stages = sorted({s.stage_id for s in plan.stages if s.replica_id == stage.replica_id})
    if micro == 0:
        return 0
    return estimate_memory(
        c, tp_degree=stage.tp_degree, stage_layers=stage.stage_layers, micro_batches=micro,
        sequence_length=c.seq_len, vocab_size=c.vocab_size,
        in_flight_micro_batches=peak_in_flight(micro, stage_index=stages.index(stage.stage_id),
                                               num_stages=len(stages)),
    ).total


def describe(plan) -> dict:
    """The summary line of one plan."""
    per_replica = Counter(r for r, _mb in {(p.replica_id, p.micro_batch) for p in plan.placements})
    memory = max((_stage_memory(plan, s) for s in plan.stages), default=0)
    return {
        "version": plan.version, "step": plan.step, "digest": plan.digest,
        "failed_ranks": list(plan.failed_ranks), "active_ranks": list(plan.active_ranks),
        "stages": [{"replica": s.replica_id, "stage": s.stage_id, "tp_members": list(s.tp_members),
                    "layers": list(s.layer_range)} for s in plan.stages],
        "micro_batches": {str(r): n for r, n in sorted(per_replica.items())},
        "routes": dict(sorted(Counter(r.reshard for r in plan.state_routes).items())),
        "memory": {"max_rank_bytes": memory, "budget_bytes": plan.config.memory_budget_bytes},
    }


def plans(config, failures):
    """Yield ``{"plan": ...}`` per plan of the schedule, ending with ``{"stopped": ...}``
    if the planner stops it."""
    kw = dict(memory_budget=config.memory_budget_bytes, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    plan = build_plan(config, step=0, version=0, **kw)
    yield {"plan": describe(plan)}
    failed: list[int] = []
    for event in failures:
        failed.append(event.failed_rank)
        try:
            plan = build_plan(config, step=event.after_iteration, version=plan.version + 1,
                              failed_ranks=tuple(failed), previous=plan, **kw)
        except InfeasiblePlan as error:
            yield {"stopped": error.reason.code, "reason": error.reason.message,
                   "after_iteration": event.after_iteration}
            return
        yield {"plan": describe(plan)}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description="print the plans a training config and failure schedule produce")
    p.add_argument("--config", required=True, type=Path)
    p.add_argument("--failures", type=Path, default=None)
    args = p.parse_args(argv)
    if args.failures is None:
        train, failures = parse_train(json.loads(args.config.read_text(encoding="utf-8"))), ()
    else:
        loaded = load_config(args.config, args.failures)
        train, failures = loaded.train, loaded.failures
    for line in plans(train, failures):
        print(json.dumps(line, ensure_ascii=False), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
