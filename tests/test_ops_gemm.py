"""tcgen05 GEMM numerics against an FP32 torch reference of the same product."""

import pytest
import torch

from resihp import ops
from resihp.ops import _ext

pytestmark = pytest.mark.gpu

SHAPES = [
    (128, 128, 64),
    (256, 384, 128),
    (300, 200, 136),      # ragged M/N/K edges
    (1024, 2048, 512),
    (4096, 6144, 2048),
]


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_forward_dgrad_wgrad(m, n, k):
    torch.manual_seed(0)
    x = torch.randn(m, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") / k**0.5).bfloat16()
    dy = torch.randn(m, n, device="cuda").bfloat16()
    y = ops.linear(x, w)
    ref = x.float() @ w.float().t()
    assert _rel(y, ref) < 1e-2
    dx = ops.linear_dgrad(dy, w)
    assert _rel(dx, dy.float() @ w.float()) < 1e-2
    dw = ops.linear_wgrad(dy, x)
    ref_dw = dy.float().t() @ x.float()
    assert _rel(dw, ref_dw) < 1e-3
    acc = torch.ones_like(dw)
    ops.linear_wgrad(dy, x, out=acc, accumulate=True)
    assert _rel(acc, ref_dw + 1) < 1e-3
    ops.check_device_errors()


def test_residual_epilogue_and_both_tiles():
    torch.manual_seed(1)
    x = torch.randn(512, 256, device="cuda").bfloat16()
    w = (torch.randn(1024, 256, device="cuda") / 16).bfloat16()
    r = torch.randn(512, 1024, device="cuda").bfloat16()
    ref = x.float() @ w.float().t() + r.float()
    for bn in (128, 256):
        out = torch.empty(512, 1024, device="cuda", dtype=torch.bfloat16)
        _ext.require().gemm(x, False, w, False, out, 3, 1.0, r, 0, bn)
        assert _rel(out, ref) < 1e-2
    # a tiny grid forces many tiles per CTA through both TMEM accumulators
    out = torch.empty(512, 1024, device="cuda", dtype=torch.bfloat16)
    _ext.require().gemm(x, False, w, False, out, 0, 1.0, None, 3, 128)
    assert _rel(out, x.float() @ w.float().t()) < 1e-2
    ops.check_device_errors()


@pytest.mark.parametrize("m,n,k", [(256, 256, 64), (300, 520, 136), (1024, 2048, 512), (4096, 2048, 5504),
                                   (512, 512, 8192)])
def test_cta_pair_tiles(m, n, k):
    """The 256 x 256 CTA-pair kernel (force_bn=512) against FP32 torch, for the forward,
    dgrad and wgrad operand layouts and every epilogue the linear layers use, next to the
    single-CTA kernel (force_bn=256); a one-pair grid pushes many tiles through both
    TMEM accumulators; 512 x 512 x 8192 is four tiles of 128 K blocks each."""
    torch.manual_seed(2)
    lib = _ext.require()
    x = torch.randn(m, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") / k**0.5).bfloat16()
    dy = torch.randn(m, n, device="cuda").bfloat16()
    r = torch.randn(m, n, device="cuda").bfloat16()
    fwd = x.float() @ w.float().t()
    cases = [
        # (A, a_mn, B, b_mn, epilogue, out dtype, out shape, residual, reference)
        (x, False, w, False, 0, torch.bfloat16, (m, n), None, fwd),
        (x, False, w, False, 3, torch.bfloat16, (m, n), r, fwd + r.float()),
        (dy, False, w, True, 0, torch.bfloat16, (m, k), None, dy.float() @ w.float()),
        (dy, False, w, True, 1, torch.float32, (m, k), None, dy.float() @ w.float()),
        (dy, True, x, True, 1, torch.float32, (n, k), None, dy.float().t() @ x.float()),
    ]
    for a, a_mn, b, b_mn, epi, dtype, shape, res, ref in cases:
        for bn, max_ctas in ((256, 0), (512, 0), (512, 2)):
            out = torch.empty(shape, device="cuda", dtype=dtype)
            lib.gemm(a, a_mn, b, b_mn, out, epi, 1.0, res, max_ctas, bn)
            assert _rel(out, ref) < 1e-2, (epi, bn, max_ctas)
    # accumulating wgrad epilogues (load-add-store and red.global.add)
    ref_dw = dy.float().t() @ x.float()
    for epi in (2, 4):
        acc = torch.ones(n, k, device="cuda")
        lib.gemm(dy, True, x, True, acc, epi, 1.0, None, 0, 512)
        assert _rel(acc, ref_dw + 1) < 1e-3
    ops.check_device_errors()
