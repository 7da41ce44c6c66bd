"""The weight-gradient GEMM's ``red.global.add`` epilogue (the default; ``RESIHP_WGRAD_RED=0`` turns it off).

Accumulating ``dy^T x`` into an FP32 buffer through fire-and-forget L2 reductions must
give exactly the sums of the load-add-store epilogue (each element receives one
addition per launch; the data here has no subnormals), on a shape with a partial tile
and on the 1.3B QKV shape. Runs last in the GPU tier.
"""

import pytest
import torch

from resihp.ops import _ext, check_device_errors
from resihp.ops.gemm import EPI_ACC_F32, EPI_RED_F32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k", [(384, 200, 136), (4096, 6144, 2048)])
def test_red_epilogue_equals_load_add_store(m, n, k):
    torch.manual_seed(0)
    dy = torch.randn(m, n, device="cuda").bfloat16()
    x = torch.randn(m, k, device="cuda").bfloat16()
    start = torch.randn(n, k, device="cuda")
    a, b = start.clone(), start.clone()
    lib = _ext.require()
    for _ in range(2):
        lib.gemm(dy, True, x, True, a, EPI_ACC_F32)
        lib.gemm(dy, True, x, True, b, EPI_RED_F32)
    torch.cuda.synchronize()
    check_device_errors(0)
    assert torch.equal(a, b)
    ref = start + 2 * (dy.float().t() @ x.float())
    assert ((a - ref).norm() / ref.norm()).item() < 1e-3
