"""Small single-GPU workloads of the hot kernels, sized for profiler captures.

    python bench_kernels.py gemm   # forward + wgrad GEMM, 4096 x 6144 x 2048
    python bench_kernels.py attn   # causal attention fwd + bwd, B2 H16 S2048 D128
    python bench_kernels.py dp     # fused DP all-reduce + AdamW, 2 replicas emulated, 64M elements
    python bench_kernels.py reshard  # state move TP2 -> TP1 of one 1.3B layer group (3 fields)
    python bench_kernels.py gemm_time  # CUDA-event TF/s: forward / dgrad / wgrad / cuBLAS forward
    python bench_kernels.py attn_time  # CUDA-event fwd / bwd time of the causal attention
    python bench_kernels.py fused_ag [tp]  # fused AG->GEMM, 1.3B QKV shape, peers emulated locally
    python bench_kernels.py fused_rs [tp]  # fused GEMM->RS, 1.3B down-proj shape, peers emulated
    python bench_kernels.py fused_ar [tp]  # fused GEMM->AR (no sequence parallelism), same shape
    python bench_kernels.py fused_time  # CUDA-event time of the emulated fused kernels vs the GEMM alone
    python bench_kernels.py mem_time  # achieved GB/s of RMSNorm, RoPE, SwiGLU and AdamW

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


def _time_us(fn_, it: int = 20, warm: int = 5) -> float:
    """CUDA-event time of one call (``warm`` untimed calls, then ``it`` timed back to back)."""
    for _ in range(warm):
        fn_()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(it):
        fn_()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / it * 1000.0


def gemm_time() -> None:
    """TF/s of the three linear-layer products (the weight gradient accumulated by
    load-add-store and by ``red.global.add``) and of ``torch.matmul`` on the 1.3B shapes."""
    import json

    out = []
    for m, n, k in ((4096, 6144, 2048), (4096, 11008, 2048), (4096, 2048, 5504), (8192, 8192, 8192)):
        x = torch.randn(m, k, device="cuda").bfloat16()
        w = torch.randn(n, k, device="cuda").bfloat16()
        dy = torch.randn(m, n, device="cuda").bfloat16()
        acc = torch.zeros(n, k, device="cuda")
        flop = 2.0 * m * n * k
        row = {"m": m, "n": n, "k": k}
        k_ = ops._ext.require()
        for name, fn_ in (("forward", lambda: ops.linear(x, w)), ("dgrad", lambda: ops.linear_dgrad(dy, w)),
                          ("wgrad", lambda: k_.gemm(dy, True, x, True, acc, 2)),
                          ("wgrad_red", lambda: k_.gemm(dy, True, x, True, acc, 4)),
                          ("cublas_forward", lambda: torch.matmul(x, w.t()))):
            row[name + "_tflops"] = round(flop / _time_us(fn_) / 1e6, 1)
        out.append(row)
    print(json.dumps(out))


def attn_time() -> None:
    """Forward and backward time of the causal attention at B2 H16 S2048 D128."""
    import json

    seq, hq, d, b = 2048, 16, 128, 2
    k = ops._ext.require()
    qkv = torch.randn(b * seq, 3 * hq * d, device="cuda").bfloat16()
    out, lse = k.attn_fwd(qkv, seq, hq, hq, d, d**-0.5)
    dout = torch.randn_like(out)
    fwd = _time_us(lambda: k.attn_fwd(qkv, seq, hq, hq, d, d**-0.5))
    bwd = _time_us(lambda: k.attn_bwd(qkv, out, dout, lse, seq, hq, hq, d, d**-0.5))
    flop = 2 * 2 * b * hq * seq * seq * d / 2  # two products, causal half
    print(json.dumps({"fwd_us": round(fwd, 1), "bwd_us": round(bwd, 1), "fwd_tflops": round(flop / fwd / 1e6, 1),
                      "bwd_tflops": round(2.5 * flop / bwd / 1e6, 1)}))


def dp() -> None:
    """One DP rank of two; the peer's region is a second local region (flags preset)."""
    from resihp.models.layout import TensorSpec
    from resihp.parallel.tp import FlatState

    k = ops._ext.require()
    n = 64 * 1024 * 1024
    dev = torch.device("cuda", 0)
    a, b = (FlatState([(TensorSpec("w", (n,), None, "normal"), (n,))], dev, torch.bfloat16, shared=True)
            for _ in range(2))
    for f in (a, b):
        f.grads[0].normal_()
    a.exp_avg_sq.fill_(1e-4)
    grid = k.dp_grid(n, 0)
    a.flags.view(-1, 8)[:grid, 1] = 1 << 20
    for step in range(1, 4):
        k.dp_allreduce_adamw([a.grads[0].data_ptr(), b.grads[0].data_ptr()], 0, a.grads[1], a.master, a.exp_avg,
                             a.exp_avg_sq, a.work, 1e-4, 0.9, 0.95, 1e-8, 0.1, step, 1.0, a.region_ptr,
                             [a.region_ptr, b.region_ptr], step, grid)


def reshard() -> None:
    """Two TP2 donors -> one TP1 target: q/k/v + gate/up (dim 0), o/down (dim 1), norms."""
    from resihp.models.layout import TensorSpec
    from resihp.parallel.peer import GatherPlan, shard_pieces
    from resihp.parallel.tp import FlatState, local_slice

    dev = torch.device("cuda", 0)
    d, f = 2048, 5504
    logical = [("qkv", (3 * d, d), 0), ("o", (d, d), 1), ("gate_up", (2 * f, d), 0), ("down", (d, f), 1),
               ("norm", (d,), None)]

    def flat(degree, idx):
        entries = [(TensorSpec(n, s, dim, "normal"), tuple(local_slice(torch.empty(s), dim, idx, degree).shape))
                   for n, s, dim in logical]
        return FlatState(entries, dev, torch.bfloat16, shared=True)

    donors = [flat(2, i) for i in range(2)]
    for x in donors:
        x.master.normal_()
    target = flat(1, 0)
    for _ in range(3):
        gp = GatherPlan()
        for name, s, dim in logical:
            for piece in shard_pieces(s, dim, 2, 1, 0):
                src = donors[piece.donor]
                gp.add([piece], src_region=src.region_ptr, src_fields=src.field_offsets,
                       src_tensor_off=src.offsets[name][0], dst_flat=target, dst_tensor_off=target.offsets[name][0])
        gp.launch(dev)


def fused_ag(tp: int = 2) -> None:
    """Three emulated AG->GEMM launches at the 1.3B QKV shape (T 4096, K 2048, N 6144/tp)."""
    from resihp.utils.fused_emulation import AgSession

    s = AgSession(4096, 2048, 3 * 2048 // tp, tp=tp)
    for _ in range(3):
        s.launch()


def fused_rs(tp: int = 2, all_reduce: bool = False) -> None:
    """Three emulated GEMM->RS (or GEMM->AR) launches at the 1.3B down-projection shape."""
    from resihp.utils.fused_emulation import RsSession

    s = RsSession(4096, 5504 // tp, 2048, tp=tp, all_reduce=all_reduce)
    for _ in range(3):
        s.launch()


def mem_time() -> None:
    """Achieved bandwidth of the memory-bound step kernels at the 1.3B micro-batch shapes
    (4096 tokens, d 2048, FFN 5504, 32 rotated Q/K heads of 128): algorithmic bytes (each
    input read once, each output written once) over the CUDA-event time, and the fraction
    of the measured copy bandwidth. Three sets of buffers are used in turn, so consecutive
    calls never find their inputs in the 126 MB L2."""
    import json
    import os

    peaks = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    hbm = json.load(open(peaks))["hbm_gbs"] if os.path.exists(peaks) else None
    t, d, f, heads, hd, seq = 4096, 2048, 5504, 32, 128, 2048
    k = ops._ext.require()
    w = (1 + 0.1 * torch.randn(d, device="cuda")).bfloat16()
    dw = torch.zeros(d, device="cuda")
    cs = fn.rope_table(seq, hd, 10000.0, device="cuda")
    sets = []
    for _ in range(3):
        x, r = (torch.randn(t, d, device="cuda").bfloat16() for _ in range(2))
        y, s, rstd = k.rmsnorm_fwd(x, r, w, 1e-5)
        sets.append({"x": x, "r": r, "s": s, "rstd": rstd, "dy": torch.randn_like(x), "dres": torch.randn_like(x),
                     "qkv": torch.randn(t, 3 * d, device="cuda").bfloat16(),
                     "gu": torch.randn(t, 2 * f, device="cuda").bfloat16(),
                     "dh": torch.randn(t, f, device="cuda").bfloat16()})
    n = 64 * 2**20
    flat = [torch.randn(n, device="cuda") for _ in range(4)]
    pb = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    act = t * d * 2
    cases = {
        "rmsnorm_fwd_residual": (lambda b: k.rmsnorm_fwd(b["x"], b["r"], w, 1e-5), 4 * act),
        "rmsnorm_bwd_residual": (lambda b: k.rmsnorm_bwd(b["dy"], b["s"], w, b["rstd"], b["dres"], dw, True), 4 * act),
        "rope_qk": (lambda b: k.rope(b["qkv"], cs, seq, heads, hd, 0, False), 2 * t * heads * hd * 2),
        "swiglu_fwd": (lambda b: k.swiglu_fwd(b["gu"]), 3 * t * f * 2),
        "swiglu_bwd": (lambda b: k.swiglu_bwd(b["gu"], b["dh"]), 5 * t * f * 2),
    }
    out = []
    for name, (call, nbytes) in cases.items():
        i = [0]

        def rotate():
            call(sets[i[0] % 3])
            i[0] += 1

        us = _time_us(rotate, it=30, warm=6)
        row = {"kernel": name, "us": round(us, 2), "gbs": round(nbytes / us / 1e3, 1)}
        if hbm:
            row["of_measured_hbm"] = round(nbytes / us / 1e3 / hbm, 3)
        out.append(row)
    # AdamW over 64 Mi fp32 elements: p, g, m, v read, p, m, v written, bf16 copy written
    us = _time_us(lambda: k.adamw(flat[0], flat[1], flat[2], flat[3], pb, 1e-4, 0.9, 0.95, 1e-8, 0.1, 1, 1.0),
                  it=10, warm=3)
    nbytes = n * (7 * 4 + 2)
    row = {"kernel": "adamw_64Mi", "us": round(us, 1), "gbs": round(nbytes / us / 1e3, 1)}
    if hbm:
        row["of_measured_hbm"] = round(nbytes / us / 1e3 / hbm, 3)
    out.append(row)
    print(json.dumps(out))


def fused_time() -> None:
    """CUDA-event time of the fused TP kernels with the peers emulated by local buffers
    (the kernel's structure without NVLink latency) against this package's GEMM alone
    on the same shape, at TP 2, 4 and 8 (1.3B shapes)."""
    import json

    from resihp.utils.fused_emulation import AgSession, RsSession

    out = []
    for tp in (2, 4, 8):
        n_ag, k_rs = 3 * 2048 // tp, 5504 // tp
        x = torch.randn(4096, 2048, device="cuda").bfloat16()
        w = torch.randn(n_ag, 2048, device="cuda").bfloat16()
        h = torch.randn(4096, k_rs, device="cuda").bfloat16()
        w2 = torch.randn(2048, k_rs, device="cuda").bfloat16()
        ag, rs = AgSession(4096, 2048, n_ag, tp=tp), RsSession(4096, k_rs, 2048, tp=tp)
        ar = RsSession(4096, k_rs, 2048, tp=tp, all_reduce=True)
        out.append({"tp": tp, "ag_gemm_alone_us": round(_time_us(lambda: ops.linear(x, w)), 1),
                    "ag_us": round(_time_us(ag.launch), 1),
                    "rs_gemm_alone_us": round(_time_us(lambda: ops.linear(h, w2)), 1),
                    "rs_us": round(_time_us(rs.launch), 1), "ar_us": round(_time_us(ar.launch), 1)})
    print(json.dumps(out))


def main(argv=None) -> None:
    args = argv or sys.argv[1:]
    what = args[0]
    torch.manual_seed(0)
    if what in ("fused_ag", "fused_rs", "fused_ar"):
        tp = int(args[1]) if len(args) > 1 else 2
        if what == "fused_ag":
            fused_ag(tp)
        else:
            fused_rs(tp, all_reduce=what == "fused_ar")
    else:
        {"gemm": gemm, "attn": attn, "dp": dp, "reshard": reshard, "gemm_time": gemm_time,
         "attn_time": attn_time, "fused_time": fused_time, "mem_time": mem_time}[what]()
    torch.cuda.synchronize()
    ops.check_device_errors()
    print("ok", what)


if __name__ == "__main__":
    main()
