"""Measurement-only hook for timing the unmodified reference's fail-stop recovery.

Put this directory first on ``PYTHONPATH`` of the reference's launcher (with
``RESIHP_REFHOOK=1``); every worker then imports it at start-up. It changes no file of
the reference: when the reference's ``resihp.control`` module loads, it wraps
``ControlPlane.observe``, ``safe_point`` and ``training_step`` with timers and prints one
``{"refrecovery": ...}`` JSON line per fail-stop (numbered from 1; failure detected at the
boundary -> end of the first resumed step, the same interval this framework reports) and a
``{"refstep": ...}`` line per trained step. ``RESIHP_REF_VOCAB`` / ``RESIHP_REF_SEQ``
replace the reference's hard-coded run constants (vocabulary 256, sequence 16) so it
can run the config-1 shape.
"""

import importlib.abc
import importlib.machinery
import json
import os
import sys
import time


def _patch(control):
    main = sys.modules["__main__"]  # resihp.train runs as __main__ under python -m
    if hasattr(main, "VOCAB_SIZE"):
        main.VOCAB_SIZE = int(os.environ.get("RESIHP_REF_VOCAB", main.VOCAB_SIZE))
        main.SEQUENCE_LENGTH = int(os.environ.get("RESIHP_REF_SEQ", main.SEQUENCE_LENGTH))
    state = {"t_fail": None, "pending": False, "t_sp": None, "event": 0}
    cls = control.ControlPlane
    observe, safe_point, training_step = cls.observe, cls.safe_point, cls.training_step

    def timed_observe(self):
        t = time.perf_counter()
        lost = observe(self)
        if lost:
            state["t_fail"] = t
        return lost

    def timed_safe_point(self, *args, **kwargs):
        out = safe_point(self, *args, **kwargs)
        state["event"] += 1
        state["pending"] = True
        state["t_sp"] = time.perf_counter()
        return out

    def timed_training_step(self):
        t0 = time.perf_counter()
        out = training_step(self)
        t1 = time.perf_counter()
        if self.training_run is not None:
            print(json.dumps({"refstep": {"rank": self.rank, "step_s": t1 - t0}}), flush=True)
        if state["pending"]:
            state["pending"] = False
            print(json.dumps({"refrecovery": {"rank": self.rank, "event": state["event"],
                                              "seconds": t1 - state["t_fail"],
                                              "safe_point_s": state["t_sp"] - state["t_fail"],
                                              "first_step_s": t1 - t0}}), flush=True)
        return out

    cls.observe, cls.safe_point, cls.training_step = timed_observe, timed_safe_point, timed_training_step


class _Finder(importlib.abc.MetaPathFinder):
    def find_spec(self, name, path, target=None):
        if name != "resihp.control":
            return None
        spec = importlib.machinery.PathFinder.find_spec(name, path)
        if spec is None:
            return None
        execute = spec.loader.exec_module

        def exec_module(module):
            execute(module)
            _patch(module)

        spec.loader.exec_module = exec_module
        return spec


if os.environ.get("RESIHP_REFHOOK") == "1":
    sys.meta_path.insert(0, _Finder())
