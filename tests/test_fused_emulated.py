"""Fused AG->GEMM / GEMM->RS kernels on ONE GPU, peers emulated by local buffers.

The launch of group rank 0 reads "peer" chunks / partials from second buffers on the
same device whose flag words are set beforehand, so no launch waits on another (see
``resihp.utils.fused_emulation``). Results are compared with an FP32 torch product for
TP degrees 2, 4 and 8 -- the kernels' gather, tile order, per-chunk readiness and
rank-ordered reduction are all exercised without a second GPU.
"""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu

# The row-block variant (TP > 2) joins these tests once it has been measured on GPUs.
VARIANTS = [0, 1] if os.environ.get("RESIHP_FUSED_TP_V3", "0") == "1" else [0]


def _rel(a, b):
    return ((a.float() - b).norm() / b.norm()).item()


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("tp", [2, 4, 8])
def test_emulated_ag_gemm(tp, variant):
    from resihp.ops import check_device_errors
    from resihp.utils.fused_emulation import emulate_ag

    for epoch in (1, 2):
        y, ref, xg, x_full = emulate_ag(1024, 512, 768, tp=tp, epoch=epoch, seed=tp + epoch, variant=variant)
        torch.cuda.synchronize()
        check_device_errors(0)
        assert torch.equal(xg, x_full)  # the gather buffer holds the whole gathered input
        assert _rel(y, ref) < 1e-2


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("tp", [2, 4, 8])
def test_emulated_gemm_rs(tp, variant):
    from resihp.ops import check_device_errors
    from resihp.utils.fused_emulation import emulate_rs

    for epoch in (1, 2):
        y, ref = emulate_rs(1024, 512, 768, tp=tp, epoch=epoch, seed=10 * tp + epoch, variant=variant)
        torch.cuda.synchronize()
        check_device_errors(0)
        assert _rel(y, ref) < 1e-2
