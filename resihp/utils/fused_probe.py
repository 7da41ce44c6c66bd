"""Fused AG->GEMM / GEMM->RS against NCCL + GEMM at the 1.3B model's layer shapes.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \
        --master-port 29581 -m resihp.utils.fused_probe

CUDA-event timing (5 warm-up, 20 launches, max over ranks); rank 0 prints JSON.
"""

import json
import os

import torch
import torch.distributed as dist

rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl")
from resihp.parallel.fused import SymmetricWorkspace
from resihp import ops
T, d = 4096, 2048
tl = T // world
ws = SymmetricWorkspace(dist.group.WORLD, tl, d, torch.device("cuda", rank))
def t_ev(fn, it=20, warm=5):
    for _ in range(warm): fn()
    torch.cuda.synchronize(); dist.barrier()
    s = torch.cuda.Event(enable_timing=True); e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(it): fn()
    e.record(); torch.cuda.synchronize()
    v = torch.tensor([s.elapsed_time(e) / it], device="cuda"); dist.all_reduce(v, op=dist.ReduceOp.MAX)
    return v.item() * 1000
res = {}
x = torch.randn(tl, d, device="cuda").bfloat16()
for name, n in (("qkv", 3 * d // world * 1), ("gate_up", 2 * 5504 // world)):
    w = torch.randn(n, d, device="cuda").bfloat16()
    def nccl():
        xg = torch.empty(T, d, device="cuda", dtype=torch.bfloat16)
        dist.all_gather_into_tensor(xg, x)
        return ops.linear(xg, w)
    def fused():
        return ws.all_gather_gemm(x, w, False, n)
    xg_full = torch.randn(T, d, device="cuda").bfloat16()
    res[f"ag_{name}_n{n}_us"] = dict(nccl=t_ev(nccl), fused=t_ev(fused), gemm_only=t_ev(lambda: ops.linear(xg_full, w)),
                                     ag_only=t_ev(lambda: dist.all_gather_into_tensor(torch.empty(T, d, device="cuda", dtype=torch.bfloat16), x)))
for name, k in (("o", d // world), ("down", 5504 // world)):
    h = torch.randn(T, k, device="cuda").bfloat16(); w = torch.randn(d, k, device="cuda").bfloat16()
    def nccl():
        y = ops.linear(h, w); out = torch.empty(tl, d, device="cuda", dtype=torch.bfloat16)
        dist.reduce_scatter_tensor(out, y); return out
    res[f"rs_{name}_k{k}_us"] = dict(nccl=t_ev(nccl), fused=t_ev(lambda: ws.gemm_reduce_scatter(h, w, False, d)),
                                     gemm_only=t_ev(lambda: ops.linear(h, w)))
ops.check_device_errors(rank)
if rank == 0: print(json.dumps(res, indent=1))
ws.close(); dist.destroy_process_group()
