"""The driver's smoke entry point (``__graft_entry__.smoke``): one tiny forward + backward
+ AdamW step of the flagship Llama-style model through the sm_100a kernels."""

import os
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_smoke_entry_point_runs():
    sys.path.insert(0, ROOT)
    import __graft_entry__

    __graft_entry__.smoke()
