"""Experimental kernel variants that are off by default, on ONE GPU (runs last in the GPU tier).

Opt-in (``RESIHP_TEST_EXPERIMENTAL=1``) until each has run on a GPU:

* pipelined RS / AR partial-tile pushes (``RESIHP_PUSH_DEPTH=2``), peers emulated: a copy
  thread issues a partial-tile push and counts the previous one only once it has landed
  (``bulk_push_issue`` + ``cp.async.bulk.wait_group``), paying every owed count before it
  waits on a peer. The output must equal the default path's bit for bit, rank 0's
  partial tiles must reach every owner's receive buffer, and every owner's tile counter
  must be incremented exactly once per call;
* the seven-stage CTA-pair GEMM (``RESIHP_GEMM_STAGES=7``, read once per process, so it
  runs in a child process): forward, dgrad and wgrad products against FP32 torch, and
  bit for bit against the six-stage kernel (the stage count changes no arithmetic);
* the streaming RMSNorm backward (``RESIHP_NORM_STREAM=1``, child process): ds bit for
  bit equal to the register kernel's, dw equal up to the order of its fp32 row sums.
"""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(os.environ.get("RESIHP_TEST_EXPERIMENTAL") != "1",
                       reason="opt-in: set RESIHP_TEST_EXPERIMENTAL=1 to run the experimental kernel variants"),
]
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

T, K, N = 1024, 512, 768


@pytest.mark.parametrize("all_reduce", [False, True], ids=["rs", "ar"])
@pytest.mark.parametrize("tp", [2, 4])
def test_pipelined_pushes_match_the_default_path(tp, all_reduce):
    from resihp.ops import check_device_errors
    from resihp.parallel import fused
    from resihp.utils.fused_emulation import Emulation

    def run(depth):
        em = Emulation(T, N, tp=tp, seed=10 * tp)
        g = torch.Generator(device="cuda").manual_seed(5 + tp)
        hs = [torch.randn(T, K, device="cuda", generator=g).bfloat16() for _ in range(tp)]
        ws = [(torch.randn(N, K, device="cuda", generator=g) / K**0.5).bfloat16() for _ in range(tp)]
        em.preset_partials(hs, ws, all_reduce=all_reduce)
        em.kx.set_fused_push_depth(depth)
        try:
            outs = []
            for call in (1, 2):
                y = em.gemm_all_reduce(hs[0], ws[0]) if all_reduce else em.gemm_reduce_scatter(hs[0], ws[0])
                torch.cuda.synchronize()
                check_device_errors(0)
                per_chunk = (em.rpr // 128) * ((N + 255) // 256)
                for owner in range(1, tp):
                    bank = em.u32(owner, fused._RS_CNT, 2 * fused.MAX_TILES).view(2, fused.MAX_TILES)[call % 2]
                    assert torch.equal(bank[:per_chunk].cpu(), torch.full((per_chunk,), 1, dtype=torch.int32))
                recv = [em.from_tiles(em.recv_tiles(o, call % 2, N)[0], N) for o in range(1, tp)]
                outs.append((y.clone(), [r.clone() for r in recv]))
            return outs
        finally:
            em.kx.set_fused_push_depth(1)

    base, piped = run(1), run(2)
    for (y1, r1), (y2, r2) in zip(base, piped):
        assert torch.equal(y1, y2)
        for a, b in zip(r1, r2):
            assert torch.equal(a, b)


_GEMM_CHILD = r"""
import hashlib, json, torch
from resihp import ops
torch.manual_seed(0)
out = {}
for m, n, k in ((4096, 6144, 2048), (4096, 2048, 5504), (1024, 768, 512)):
    x = torch.randn(m, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") / k ** 0.5).bfloat16()
    dy = torch.randn(m, n, device="cuda").bfloat16()
    y = ops.linear(x, w)
    dx = ops.linear_dgrad(dy, w)
    dw = torch.zeros(n, k, device="cuda")
    ops.linear_wgrad(dy, x, out=dw, accumulate=True)
    torch.cuda.synchronize()
    ops.check_device_errors()
    rel = lambda a, b: ((a.float() - b).norm() / b.norm()).item()
    out[f"{m}x{n}x{k}"] = {
        "rel": [rel(y, x.float() @ w.float().t()), rel(dx, dy.float() @ w.float()), rel(dw, dy.float().t() @ x.float())],
        "sha": [hashlib.sha256(t.contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()
                for t in (y.view(torch.int16), dx.view(torch.int16), dw.view(torch.int32))],
    }
print(json.dumps(out))
"""


def _gemm_child(stages):
    env = dict(os.environ, PYTHONPATH=ROOT, RESIHP_GEMM_STAGES=str(stages))
    out = subprocess.run([sys.executable, "-c", _GEMM_CHILD], cwd=ROOT, env=env, capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


def test_seven_stage_pair_gemm_matches_six_stages():
    six, seven = _gemm_child(6), _gemm_child(7)
    for shape, got in seven.items():
        assert all(r < 1e-2 for r in got["rel"]), (shape, got["rel"])
        assert got["sha"] == six[shape]["sha"], shape


_NORM_CHILD = r"""
import hashlib, json, torch
from resihp.ops import _ext
k = _ext.require()
torch.manual_seed(0)
out = {}
for rows, d in ((4096, 2048), (333, 1024), (1000, 256)):
    x = torch.randn(rows, d, device="cuda").bfloat16()
    r = torch.randn(rows, d, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(d, device="cuda")).bfloat16()
    y, s, rstd = k.rmsnorm_fwd(x, r, w, 1e-5)
    dy, dres = torch.randn_like(x), torch.randn_like(x)
    dw = torch.zeros(d, device="cuda")
    ds = k.rmsnorm_bwd(dy, s, w, rstd, dres, dw, True)
    torch.cuda.synchronize()
    out[f"{rows}x{d}"] = {"ds": hashlib.sha256(ds.view(torch.int16).cpu().numpy().tobytes()).hexdigest(),
                          "dw": dw.cpu().tolist()}
print(json.dumps(out))
"""


def _norm_child(stream):
    env = dict(os.environ, PYTHONPATH=ROOT, RESIHP_NORM_STREAM="1" if stream else "0")
    out = subprocess.run([sys.executable, "-c", _NORM_CHILD], cwd=ROOT, env=env, capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


def test_streaming_norm_backward_matches_the_register_kernel():
    base, stream = _norm_child(False), _norm_child(True)
    for shape, got in stream.items():
        assert got["ds"] == base[shape]["ds"], shape
        a, b = torch.tensor(got["dw"]), torch.tensor(base[shape]["dw"])
        assert ((a - b).norm() / b.norm()).item() < 1e-5, shape
