"""Small single-GPU workloads of the hot kernels, sized for profiler captures.

    python -m resihp.utils.kernel_probe gemm   # forward + wgrad GEMM, 4096 x 6144 x 2048
    python -m resihp.utils.kernel_probe attn   # causal attention fwd + bwd, B2 H16 S2048 D128

Each workload touches a few hundred MB (more than the 126 MB L2, far below the device)
and launches every kernel a handful of times, so a capture of one or two launches ends
by itself in a minute or two.
"""

from __future__ import annotations

import sys

import torch

from resihp import ops
from resihp.ops import functional as fn


def gemm() -> None:
    m, n, k = 4096, 6144, 2048
    x = torch.randn(m, k, device="cuda").bfloat16()
    w = torch.randn(n, k, device="cuda").bfloat16()
    dy = torch.randn(m, n, device="cuda").bfloat16()
    out = torch.zeros(n, k, device="cuda")
    for _ in range(3):
        ops.linear(x, w)
        ops.linear_wgrad(dy, x, out=out, accumulate=True)


def attn() -> None:
    seq, hq, d, b = 2048, 16, 128, 2
    cs = fn.rope_table(seq, d, 10000.0, device="cuda")
    for _ in range(2):
        qkv = torch.randn(b * seq, 3 * hq * d, device="cuda").bfloat16().requires_grad_()
        out = fn.rope_attention(qkv, cs, seq, hq, hq, d)
        out.backward(torch.randn_like(out))


def main(argv=None) -> None:
    what = (argv or sys.argv[1:])[0]
    torch.manual_seed(0)
    {"gemm": gemm, "attn": attn}[what]()
    torch.cuda.synchronize()
    ops.check_device_errors()
    print("ok", what)


if __name__ == "__main__":
    main()
