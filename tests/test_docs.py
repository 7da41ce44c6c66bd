"""The README's switch table stays in step with the code.

Every ``RESIHP_*`` environment variable the Python package or the benchmarks read with
``os.environ`` is listed in the README (the launcher's own store variables and the
reference timing hook's variables are internal plumbing and exempt).
"""

import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INTERNAL = {"RESIHP_STORE_HOST", "RESIHP_STORE_PORT", "RESIHP_REFHOOK", "RESIHP_REF_SEQ", "RESIHP_REF_VOCAB"}
READ = re.compile(r"""os\.environ(?:\.get)?[\[(]\s*["'](RESIHP_[A-Z0-9_]+)["']""")


def test_every_switch_is_documented():
    used = set()
    paths = [os.path.join(ROOT, "bench.py"), os.path.join(ROOT, "bench_recovery.py")]
    for base, _dirs, files in os.walk(os.path.join(ROOT, "resihp")):
        paths += [os.path.join(base, f) for f in files if f.endswith(".py")]
    for path in paths:
        with open(path, encoding="utf-8") as f:
            used |= set(READ.findall(f.read()))
    with open(os.path.join(ROOT, "README.md"), encoding="utf-8") as f:
        documented = set(re.findall(r"`(RESIHP_[A-Z0-9_]+)`", f.read()))
    assert used, "no switches found: the pattern is stale"
    missing = sorted(used - INTERNAL - documented)
    assert not missing, missing
