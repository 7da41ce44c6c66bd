"""Differential oracle: this planner against the reference planner, digest for digest.

The reference installed under ``baseline/_ref`` is run in a subprocess (both packages
are named ``resihp``), on the same random scenarios, and every plan digest and stop code
along each failure sequence must agree. Skipped when the reference is not installed
(a failure instead with ``RESIHP_REQUIRE_REFERENCE=1``).
"""

import json
import os
import subprocess
import sys

import pytest

import plan_scenarios
from resihp import config as our_config
from resihp import plan as our_plan

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
COUNT = 300

_WORKER = """
import json, sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(1, sys.argv[2])
import plan_scenarios
from resihp import config, plan
print(json.dumps([plan_scenarios.replay(config, plan, s) for s in plan_scenarios.scenarios(int(sys.argv[3]))]))
"""


@pytest.mark.reference
def test_digests_match_reference_planner():
    tests_dir = os.path.dirname(os.path.abspath(__file__))
    env = {k: v for k, v in os.environ.items() if k != "PYTHONPATH"}
    out = subprocess.run(
        [sys.executable, "-c", _WORKER, REF, tests_dir, str(COUNT)],
        capture_output=True, text=True, check=True, env=env, cwd="/",
    )
    theirs = json.loads(out.stdout)
    ours = [plan_scenarios.replay(our_config, our_plan, s) for s in plan_scenarios.scenarios(COUNT)]
    stops = sum(1 for t in ours if t[-1][0] == "stop")
    assert stops > 10  # the scenarios really reach infeasibility
    for index, (a, b) in enumerate(zip(ours, theirs)):
        assert a == b, (index, plan_scenarios.scenarios(COUNT)[index], a, b)
