"""Acceptance-level properties of the shipped run and of the failure model.

* The shipped schedule (``configs/train.json`` + ``configs/failures.json``, five
  consecutive fail-stops on TP2 x PP2 x DP2) must exercise all three reconfiguration
  axes: some fail-stop changes a TP degree, some moves layers between stages, and some
  reroutes micro-batches between replicas (reference ``tests/test_acceptance.py:172``).
* The failure model is fail-stop only, detected from the launcher's process table at
  iteration boundaries: no identifier in the package names a heartbeat, a failure
  detector, a standby pool or a speed/straggler signal (reference
  ``tests/test_acceptance.py:51-83`` scans for the same mechanisms).
"""

import ast
import os

from resihp.config import load_config
from resihp.plan import build_plan

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BANNED = ("heartbeat", "detector", "standby", "straggler", "speed")


def _plans():
    loaded = load_config(os.path.join(ROOT, "configs", "train.json"), os.path.join(ROOT, "configs", "failures.json"))
    c = loaded.train
    plan = build_plan(c, step=0, version=0, vocab_size=c.vocab_size, sequence_length=c.seq_len)
    plans, failed = [plan], []
    for e in loaded.failures:
        failed.append(e.failed_rank)
        plan = build_plan(c, step=e.after_iteration, version=plan.version + 1, failed_ranks=failed, previous=plan,
                          vocab_size=c.vocab_size, sequence_length=c.seq_len)
        plans.append(plan)
    return plans


def _replica_of_micro_batch(plan):
    return {p.micro_batch: p.replica_id for p in plan.placements}


def test_shipped_schedule_moves_tp_pp_and_dp():
    plans = _plans()
    assert len(plans) == 6
    tp_moves = pp_moves = dp_moves = 0
    for a, b in zip(plans, plans[1:]):
        degrees_a = {(s.replica_id, s.stage_id): s.tp_degree for s in a.stages}
        degrees_b = {(s.replica_id, s.stage_id): s.tp_degree for s in b.stages}
        tp_moves += any(degrees_b.get(k) not in (None, v) for k, v in degrees_a.items())
        ranges_a = {(s.replica_id, s.stage_id): s.layer_range for s in a.stages}
        ranges_b = {(s.replica_id, s.stage_id): s.layer_range for s in b.stages}
        pp_moves += any(ranges_b.get(k) not in (None, v) for k, v in ranges_a.items())
        dp_moves += _replica_of_micro_batch(a) != _replica_of_micro_batch(b)
    assert tp_moves and pp_moves and dp_moves, (tp_moves, pp_moves, dp_moves)


def test_no_identifier_names_a_non_fail_stop_mechanism():
    offenders = []
    for base, _dirs, files in os.walk(os.path.join(ROOT, "resihp")):
        for name in files:
            if not name.endswith(".py"):
                continue
            path = os.path.join(base, name)
            with open(path, encoding="utf-8") as f:
                tree = ast.parse(f.read(), path)
            for node in ast.walk(tree):
                ident = None
                if isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef, ast.ClassDef)):
                    ident = node.name
                elif isinstance(node, ast.Name):
                    ident = node.id
                elif isinstance(node, ast.Attribute):
                    ident = node.attr
                elif isinstance(node, ast.arg):
                    ident = node.arg
                if ident and any(word in ident.lower() for word in BANNED):
                    offenders.append(f"{os.path.relpath(path, ROOT)}:{node.lineno}:{ident}")
    assert not offenders, offenders
