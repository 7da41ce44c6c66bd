"""Fused AG->GEMM / GEMM->RS / GEMM->AR against NCCL + GEMM, on 2-8 GPUs.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port 29581 bench_fused_tp.py            # 1.3B layer shapes (T=4096, d=2048)
    ... bench_fused_tp.py --sweep                         # BASELINE config-5 sweep
    ... bench_fused_tp.py --config3                       # Llama-3-8B layer shapes
    ... bench_fused_tp.py --trace DIR                     # also: per-CTA timelines of one
                                                          # fused call per op (JSON per rank)
    RESIHP_PUSH_DEPTH=2 python -m torch.distributed.run ... bench_fused_tp.py
                                                          # RS / AR pushes pipelined two deep

The sweep covers M = 4096..32768 tokens with K, N in {5120, 13824}: column-parallel
AG->GEMM ``[M, 5120] x [5120, N/tp]`` (N = 5120, 13824) and row-parallel GEMM->RS
``[M, K/tp] x [K/tp, 5120]`` (K = 5120, 13824), each against NCCL all-gather /
reduce-scatter with cuBLAS (``torch.matmul``) and, for reference, with this
package's GEMM. The roofline of a fused op is the slower of its FLOPs at the measured
bf16 peak and the bytes that must cross NVLink at 770 GB/s per direction.

CUDA-event timing (3 warm-up, 10 launches, max over ranks); rank 0 prints JSON.
``host_us`` is the host time to issue one fused call (the launch path, no sync).
"""

from __future__ import annotations

import json
import os
import sys

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def _peaks():
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)),
                        "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f).get("bf16_tflops", 1590.0))
    return 1590.0


def main():
    from resihp import ops
    from resihp.parallel.fused import SymmetricWorkspace

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl")
    dev = torch.device("cuda", rank)
    sweep = "--sweep" in sys.argv
    config3 = "--config3" in sys.argv
    peak = _peaks()
    trace_dir = sys.argv[sys.argv.index("--trace") + 1] if "--trace" in sys.argv else None
    kx = ops._ext.require()

    def host_us(fn, it=20):
        import time

        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(it):
            fn()
        t1 = time.perf_counter()
        torch.cuda.synchronize()
        return (t1 - t0) / it * 1e6

    def trace(name, fn):
        """One call with the per-CTA stamps on; rank r writes DIR/<name>_rank<r>.json."""
        if trace_dir is None:
            return
        slots = kx.fused_trace_slots()
        buf = torch.zeros(1024 * slots, dtype=torch.int64, device=dev)
        torch.cuda.synchronize()
        dist.barrier()
        kx.set_fused_trace(buf.data_ptr())
        fn()
        torch.cuda.synchronize()
        kx.set_fused_trace(0)
        rows = buf.view(1024, slots).cpu().tolist()
        os.makedirs(trace_dir, exist_ok=True)
        with open(os.path.join(trace_dir, f"{name}_rank{rank}.json"), "w") as f:
            json.dump([r for r in rows if r[0] > 0], f)

    def t_ev(fn, it=10, warm=3):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(it):
            fn()
        e.record()
        torch.cuda.synchronize()
        v = torch.tensor([s.elapsed_time(e) / it], device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        return v.item() * 1000

    def roofline(flops, link_bytes):
        return max(flops / (peak * 1e12), link_bytes / (LINK_GBS * 1e9)) * 1e6

    if sweep:
        width = 5120
        ms = (4096, 8192, 16384, 32768)
        ag_ns, rs_ks = (5120, 13824), (5120, 13824)
    elif config3:  # Llama-3-8B layer shapes: QKV with 8 KV heads, gate/up, O, down; one 4096-token micro-batch
        width = 4096
        ms = (4096,)
        ag_ns, rs_ks = (4096 + 2 * 1024, 2 * 14336), (4096, 14336)
    else:
        width = 2048
        ms = (4096,)
        ag_ns, rs_ks = (3 * 2048, 2 * 5504), (2048, 5504)
    out = []
    for m in ms:
        tl = m // world
        ws = SymmetricWorkspace(dist.group.WORLD, tl, width, dev)
        x = torch.randn(tl, width, device=dev).bfloat16()
        for n_full in ag_ns:
            n = n_full // world
            w = (torch.randn(n, width, device=dev) / width**0.5).bfloat16()
            xg_buf = torch.empty(m, width, device=dev, dtype=torch.bfloat16)

            def nccl_cublas():
                dist.all_gather_into_tensor(xg_buf, x)
                return torch.matmul(xg_buf, w.t())

            def nccl_ours():
                dist.all_gather_into_tensor(xg_buf, x)
                return ops.linear(xg_buf, w)

            row = dict(op="ag_gemm", m=m, k=width, n=n_full, n_per_rank=n, tp=world,
                       fused_us=t_ev(lambda: ws.all_gather_gemm(x, w, False, n)),
                       nccl_cublas_us=t_ev(nccl_cublas), nccl_ours_us=t_ev(nccl_ours),
                       gemm_only_us=t_ev(lambda: ops.linear(xg_buf, w)),
                       host_us=host_us(lambda: ws.all_gather_gemm(x, w, False, n)))
            trace(f"ag_{m}_{n_full}", lambda: ws.all_gather_gemm(x, w, False, n))
            row["roofline_us"] = roofline(2.0 * m * width * n, (world - 1) / world * m * width * 2)
            out.append(row)
        for k_full in rs_ks:
            k = k_full // world
            h = torch.randn(m, k, device=dev).bfloat16()
            w = (torch.randn(width, k, device=dev) / k**0.5).bfloat16()
            y_buf = torch.empty(tl, width, device=dev, dtype=torch.bfloat16)

            def nccl_cublas():
                y = torch.matmul(h, w.t())
                dist.reduce_scatter_tensor(y_buf, y)
                return y_buf

            def nccl_ours():
                y = ops.linear(h, w)
                dist.reduce_scatter_tensor(y_buf, y)
                return y_buf

            row = dict(op="gemm_rs", m=m, k=k_full, k_per_rank=k, n=width, tp=world,
                       fused_us=t_ev(lambda: ws.gemm_reduce_scatter(h, w, False, width)),
                       nccl_cublas_us=t_ev(nccl_cublas), nccl_ours_us=t_ev(nccl_ours),
                       gemm_only_us=t_ev(lambda: ops.linear(h, w)),
                       host_us=host_us(lambda: ws.gemm_reduce_scatter(h, w, False, width)))
            trace(f"rs_{m}_{k_full}", lambda: ws.gemm_reduce_scatter(h, w, False, width))
            row["roofline_us"] = roofline(2.0 * m * k * width, (world - 1) / world * m * width * 2)
            out.append(row)
            if sweep:
                continue

            def nccl_cublas_ar():
                y = torch.matmul(h, w.t())
                dist.all_reduce(y)
                return y

            # without sequence parallelism: the row-parallel output all-reduce
            row = dict(op="gemm_ar", m=m, k=k_full, k_per_rank=k, n=width, tp=world,
                       fused_us=t_ev(lambda: ws.gemm_all_reduce(h, w, False, width)),
                       nccl_cublas_us=t_ev(nccl_cublas_ar), gemm_only_us=t_ev(lambda: ops.linear(h, w)),
                       host_us=host_us(lambda: ws.gemm_all_reduce(h, w, False, width)))
            trace(f"ar_{m}_{k_full}", lambda: ws.gemm_all_reduce(h, w, False, width))
            row["roofline_us"] = roofline(2.0 * m * k * width, 2 * (world - 1) / world * m * width * 2)
            out.append(row)
        ws.close()
        del x
        torch.cuda.empty_cache()
    ops.check_device_errors(rank)
    if rank == 0:
        for row in out:
            for key in list(row):
                if key.endswith("_us"):
                    row[key] = round(row[key], 1)
            row["fused_vs_nccl_cublas"] = round(row["nccl_cublas_us"] / row["fused_us"], 3)
            row["fused_fraction_of_roofline"] = round(row["roofline_us"] / row["fused_us"], 3)
            print(json.dumps(row), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
