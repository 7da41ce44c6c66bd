"""The command-line surface: worker echo mode, launcher verdicts, membership publication.

* ``python -m resihp.train`` without ``RANK`` echoes both files as one sorted JSON line
  (reference ``resihp/train.py:180-192``);
* the launcher rejects an invalid config before spawning anything, and its verdict is
  0 only when exactly the scheduled ranks died of SIGKILL (reference
  ``resihp/launch.py:85-106``);
* the supervisor publishes a boundary's membership once every live process arrived, and
  a process that exited is left out (reference ``resihp/membership.py:134-163``).
"""

import json
import os
import subprocess
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CONFIG = os.path.join(ROOT, "configs", "train.json")
FAILURES = os.path.join(ROOT, "configs", "failures.json")


def _run(args, **kw):
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    env["PYTHONPATH"] = ROOT
    return subprocess.run([sys.executable, "-m", *args], capture_output=True, text=True, env=env, timeout=120, **kw)


def test_worker_echoes_config_without_rank():
    out = _run(["resihp.train", "--config", CONFIG, "--failures", FAILURES])
    assert out.returncode == 0, out.stderr
    line = json.loads(out.stdout)
    with open(CONFIG) as f:
        assert line["config"] == json.load(f)
    with open(FAILURES) as f:
        assert line["failures"] == json.load(f)
    assert out.stdout.strip() == json.dumps(line, ensure_ascii=False, sort_keys=True)


def test_launcher_rejects_invalid_config(tmp_path):
    bad = tmp_path / "train.json"
    with open(CONFIG) as f:
        cfg = json.load(f)
    cfg["tp"] = 0
    bad.write_text(json.dumps(cfg))
    out = _run(["resihp.launch", "--config", str(bad), "--failures", FAILURES])
    assert out.returncode != 0
    assert "tp" in out.stderr
    assert '"launch"' not in out.stdout  # nothing was spawned


def test_launcher_verdict(monkeypatch, capsys):
    from resihp import launch

    cases = [
        ({0: 0, 1: -9, 2: 0}, [1], 0),   # exactly the scheduled rank was killed
        ({0: 0, 1: 0, 2: 0}, [1], 1),    # the scheduled kill did not happen
        ({0: -9, 1: -9, 2: 0}, [1], 1),  # an unscheduled rank died
        ({0: 0, 1: -9, 2: 3}, [1], 1),   # a survivor failed
    ]
    for codes, scheduled, want in cases:
        monkeypatch.setattr(launch, "launch", lambda *a, c=codes, s=scheduled, **k: (c, s))
        assert launch.main(["--config", CONFIG, "--failures", FAILURES]) == want
        line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
        assert line["launch"]["killed_ranks"] == sorted(r for r, c in codes.items() if c == -9)


def _sleeper(seconds):
    return subprocess.Popen([sys.executable, "-c", f"import time; time.sleep({seconds})"])


def test_supervisor_publishes_membership_without_the_dead():
    from datetime import timedelta

    from resihp import membership

    sup = membership.Supervisor(range(3))
    procs = {r: _sleeper(30) for r in range(3)}
    for r, p in procs.items():
        sup.register(r, p)
    import threading

    done = {}
    t = threading.Thread(target=lambda: done.setdefault("codes", sup.serve(timeout=60)), daemon=True)
    t.start()
    try:
        procs[2].kill()  # rank 2 dies before arriving at boundary 1
        procs[2].wait()

        def arrive(rank):
            store = membership.connect(sup.host, sup.port, timedelta(seconds=30))  # one client per rank
            done[rank] = membership.boundary(store, 1, timeout=timedelta(seconds=30))

        arrivals = [threading.Thread(target=arrive, args=(r,)) for r in (0, 1)]
        for a in arrivals:
            a.start()
        for a in arrivals:
            a.join(40)
        assert done[0] == done[1] == (0, 1)
    finally:
        for p in procs.values():
            if p.poll() is None:
                p.kill()
        t.join(70)
    assert done["codes"][2] == -9
