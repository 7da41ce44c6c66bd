"""Shared pytest configuration.

``gpu`` marks every test that needs a CUDA device; the CPU tier runs with
``-m "not gpu"`` and the B200 tier with ``-m gpu``.

``reference`` marks a test that runs the unmodified reference installed under
``baseline/_ref`` (``baseline/install_reference.sh``) as an oracle. Without that install
such a test is skipped -- or fails, when ``RESIHP_REQUIRE_REFERENCE=1`` asks for the
oracle to run.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
REFERENCE = os.path.join(ROOT, "baseline", "_ref")
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    config.addinivalue_line("markers", "slow: multi-process scenario taking tens of seconds")
    config.addinivalue_line("markers", "reference: runs the reference installed under baseline/_ref as an oracle")


def pytest_runtest_setup(item):
    if item.get_closest_marker("reference") is not None and not os.path.isdir(os.path.join(REFERENCE, "resihp")):
        why = "reference not installed under baseline/_ref (bash baseline/install_reference.sh <checkout>)"
        if os.environ.get("RESIHP_REQUIRE_REFERENCE") == "1":
            pytest.fail(why)
        pytest.skip(why)


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
