"""Fused DP all-reduce + AdamW against NCCL all-reduce + the AdamW kernel, on 2+ GPUs.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29583 bench_dp_step.py [elements]

Every rank holds one flat state of ``elements`` FP32 values (default 325,000,000: one
TP2 x PP2 stage of the 1.3B model) in a shared region. CUDA-event timing (3 warm-up,
10 calls, max over ranks); rank 0 prints JSON with the roofline of the fused step: the
slower of its HBM traffic at the measured copy bandwidth and the peer gradients crossing
NVLink at 770 GB/s per direction.
"""

import json
import os
import sys

import torch
import torch.distributed as dist

from resihp.models.layout import TensorSpec
from resihp.ops import check_device_errors
from resihp.ops import functional as fn
from resihp.parallel.tp import FlatState


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    n = int(sys.argv[1]) if len(sys.argv) > 1 else 325_000_000
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl")
    dev = torch.device("cuda", rank)
    flat = FlatState([(TensorSpec("w", (n,), None, "normal"), (n,))], dev, torch.bfloat16, shared=True)
    g = torch.Generator(device="cuda").manual_seed(11 + rank)
    flat.grads[0].normal_(generator=g)
    flat.grads[1].normal_(generator=g)
    flat.master.normal_(generator=torch.Generator(device="cuda").manual_seed(3))
    flat.exp_avg_sq.fill_(1e-4)

    class _Stage:
        pass

    stage = _Stage()
    stage.flat = flat
    stage.config = type("C", (), dict(lr=1e-4, beta1=0.9, beta2=0.95, adam_eps=1e-8, weight_decay=0.1))()
    stage.use_grad = flat.set_parity
    from resihp.parallel.peer import DpPeers

    peers = DpPeers(stage, dist.group.WORLD)

    def t_ev(fn_, it=10, warm=3):
        for _ in range(warm):
            fn_()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(it):
            fn_()
        e.record()
        torch.cuda.synchronize()
        v = torch.tensor([s.elapsed_time(e) / it], device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        return v.item() * 1000

    def nccl():
        flat.step += 1
        dist.all_reduce(flat.grad)
        fn.adamw_flat(flat.master, flat.grad, flat.exp_avg, flat.exp_avg_sq, flat.step, lr=1e-4, beta1=0.9,
                      beta2=0.95, eps=1e-8, weight_decay=0.1, p_bf16=flat.work)

    fused_us = t_ev(lambda: peers.step(stage))
    nccl_us = t_ev(nccl)
    ar_us = t_ev(lambda: dist.all_reduce(flat.grad))
    adam_us = t_ev(lambda: fn.adamw_flat(flat.master, flat.grad, flat.exp_avg, flat.exp_avg_sq, 5, lr=1e-4,
                                         beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, p_bf16=flat.work))
    check_device_errors(rank)
    peaks_path = os.path.join(os.path.dirname(os.path.abspath(__file__)),
                              "MEASURED_PEAKS.json")
    hbm = 6650.0
    if os.path.exists(peaks_path):
        with open(peaks_path) as f:
            hbm = float(json.load(f).get("hbm_gbs", hbm))
    # local HBM: read g, p, m, v; write sum, p, m, v (4 B each) + bf16 copy (2 B)
    hbm_bytes = n * (4 * 4 + 4 * 4 + 2)
    link_bytes = n * 4 * (world - 1)
    target_us = max(hbm_bytes / (hbm * 1e9), link_bytes / 770e9) * 1e6
    if rank == 0:
        print(json.dumps({
            "elements": n, "world": world, "fused_us": round(fused_us, 1), "nccl_allreduce_plus_adamw_us": round(nccl_us, 1),
            "nccl_allreduce_us": round(ar_us, 1), "adamw_us": round(adam_us, 1),
            "roofline_us": round(target_us, 1), "fused_fraction_of_roofline": round(target_us / fused_us, 3),
            "hbm_gbs_used": hbm,
        }), flush=True)
    peers.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
