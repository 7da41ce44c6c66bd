"""The bounds-checked build (``-DRESIHP_BOUNDS_CHECK``, ``resihp/_C_checked.so``).

CPU: the variant is built from the same sources with the one extra define, into its own
build directory and library, and ``RESIHP_CHECKED=1`` makes the loader pick it.
GPU (runs last in the GPU tier): the checked library runs a forward GEMM, a
weight-gradient GEMM and causal attention forward + backward with every check passing
(no error recorded) and produces bit-identical results to the default library -- the
checks only test addresses, they never change the arithmetic.
"""

import json
import os
import subprocess
import sys

import pytest

from resihp.ops import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_checked_variant_is_the_same_sources_with_one_define():
    assert build.cuda_flags(checked=True) == build.CUDA_FLAGS + ["-DRESIHP_BOUNDS_CHECK"] + build.cuda_flags()[
        len(build.CUDA_FLAGS):]
    assert build.library_path(checked=True).endswith("_C_checked.so") and build.library_path().endswith("_C.so")


def test_loader_switch_names_the_checked_library():
    code = ("import json, resihp.ops._ext as e; print(json.dumps([e.CHECKED, e._LIB]))")
    for env, want in (({"RESIHP_CHECKED": "1"}, "_C_checked.so"), ({"RESIHP_CHECKED": "0"}, "_C.so")):
        out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=ROOT,
                             env={**os.environ, **env}, check=True)
        checked, lib = json.loads(out.stdout.strip().splitlines()[-1])
        assert checked == (env["RESIHP_CHECKED"] == "1") and lib.endswith(want)


_WORKLOAD = r"""
import hashlib, json, sys
import torch
from resihp.ops import _ext, check_device_errors
from resihp.ops import functional as fn
from resihp.ops.gemm import linear_wgrad
torch.manual_seed(0)
x = torch.randn(512, 256, device="cuda").bfloat16()
w = torch.randn(384, 256, device="cuda").bfloat16()
y = fn.linear(x, w)
dw = torch.zeros(384, 256, device="cuda")
linear_wgrad(y, x, out=dw, accumulate=True)
hq, hkv, d, seq = 4, 2, 128, 256
qkv = (0.5 * torch.randn(2 * seq, (hq + 2 * hkv) * d, device="cuda")).bfloat16().requires_grad_()
cs = fn.rope_table(seq, d, 10000.0, device="cuda")
o = fn.rope_attention(qkv.clone(), cs, seq, hq, hkv, d)
o.backward(torch.randn_like(o))
torch.cuda.synchronize()
check_device_errors(0)
digest = {n: hashlib.sha256(t.detach().float().cpu().numpy().tobytes()).hexdigest()
          for n, t in (("y", y), ("dw", dw), ("o", o), ("dqkv", qkv.grad))}
print(json.dumps({"lib": _ext._LIB, "digest": digest}))
"""


@pytest.mark.gpu
def test_checked_library_passes_its_checks_and_matches_bitwise():
    results = {}
    for flag in ("0", "1"):
        out = subprocess.run([sys.executable, "-c", _WORKLOAD], capture_output=True, text=True, cwd=ROOT,
                             env={**os.environ, "RESIHP_CHECKED": flag}, timeout=600)
        assert out.returncode == 0, out.stderr[-2000:]
        results[flag] = json.loads(out.stdout.strip().splitlines()[-1])
    assert results["1"]["lib"].endswith("_C_checked.so") and results["0"]["lib"].endswith("_C.so")
    assert results["1"]["digest"] == results["0"]["digest"]
