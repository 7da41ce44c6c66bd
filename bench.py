#!/usr/bin/env python
"""Headline benchmark: training tokens/s of the BASELINE config-2 model on N B200s.

Model: Llama-style 1.3B (24 layers, hidden 2048, 16 heads MHA, SwiGLU 5504, vocab 32000),
bf16 compute with FP32 master weights and AdamW; sequence 2048, micro-batch 2, global
batch 64 sequences of synthetic seeded tokens, random normal(0, 0.02) init. Layout per
N (total work fixed, so scaling is strong): below eight GPUs the fastest measured
layout, pure data parallelism (1 -> one GPU, 2 -> DP2, 4 -> DP4: 381.9k tokens/s
against 365.2k for PP2 x DP2); at eight GPUs config 2's own TP2 x PP2 x DP2 (sequence
parallel). Both arms run the same layout for each N.

``value`` is device-timed: CUDA events around exactly K steps, barrier + synchronize on
both sides, max over ranks. ``e2e`` is the same K steps through the public API
(``PlannedRun.step``: per micro-batch host-to-device copies of the tokens from pinned
memory, the loss read back to the host) timed on the host clock, max over ranks.
Every input (weights, activations, logits) is far larger than the 126 MB L2.

``--impl reference`` runs the unmodified reference from ``baseline/_ref`` through its
own public API (ControlPlane groups, ``initial_run``, ``PlannedRun.step``) at the
closest shape it can express (GPT-2 blocks, FFN 4d, FP32), printing the same line.

    python bench.py --gpus N --steps K --warmup W [--impl reference]
"""

from __future__ import annotations

import argparse
import json
import os
import socket
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "tokens/sec (device-timed, max over ranks) at 1/2/4/8 B200; fail-stop recovery seconds"
MODEL = dict(model_dim=2048, num_layers=24, num_heads=16, ffn_dim=5504, vocab_size=32000, seq_len=2048)
GLOBAL_BATCH = 64
MICRO_BATCH = 2
LAYOUTS = {1: (1, 1, 1), 2: (1, 1, 2), 4: (1, 1, 4), 8: (2, 2, 2)}  # (tp, pp, dp)

# BASELINE configs 3 and 5 (8 GPUs only; --config 3 / --config 5).
CONFIGS = {
    2: dict(model=MODEL, extra={}, global_batch=GLOBAL_BATCH, micro_batch=MICRO_BATCH, layouts=LAYOUTS,
            name="llama-1.3b (24L, d2048, 16H MHA, SwiGLU 5504, V32000)"),
    3: dict(model=dict(model_dim=4096, num_layers=32, num_heads=32, ffn_dim=14336, vocab_size=128256, seq_len=4096),
            extra=dict(num_kv_heads=8, rope_theta=500000.0), global_batch=16, micro_batch=1, layouts={8: (4, 2, 1)},
            name="llama-3-8b shape (32L, d4096, 32Q/8KV GQA, SwiGLU 14336, V128256, theta 5e5)"),
    5: dict(model=dict(model_dim=5120, num_layers=40, num_heads=40, ffn_dim=13824, vocab_size=32000, seq_len=4096),
            extra=dict(recompute=True), global_batch=8, micro_batch=1, layouts={8: (8, 1, 1)},
            name="llama-2-13b shape (40L, d5120, 40H, SwiGLU 13824, V32000), activation recompute"),
}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["resihp", "reference"], default="resihp")
    p.add_argument("--config", type=int, choices=sorted(CONFIGS), default=2,
                   help="BASELINE config: 2 (default, 1/2/4/8 GPUs), 3 or 5 (8 GPUs)")
    p.add_argument("--layout", default=None,
                   help="tp,pp,dp to run instead of the config's layout for this GPU count (e.g. 1,1,2: pure "
                        "data parallelism on 2 GPUs); the JSON line's parallelism field names what ran")
    p.add_argument("--trace", default=None,
                   help="after the timed steps, profile one more step per rank and write a Chrome trace "
                        "plus a kernel summary into this directory (analysis only; not part of the number). "
                        "With programmatic dependent launch on, a kernel's traced time includes its wait for "
                        "the previous kernel: set RESIHP_PDL=0 for per-kernel times")
    return p.parse_args()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except OSError:
            self.proc = None
            return
        threading.Thread(target=self._read, daemon=True).start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 9:
                self.rows.append(parts)

    def stop(self, visible):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        rows = [r for r in self.rows if visible is None or r[0] in visible]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def _env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def _store(rank, world):
    from torch.distributed import TCPStore

    if world == 1 and "MASTER_ADDR" not in os.environ:
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        return TCPStore("127.0.0.1", port, is_master=True, wait_for_workers=False)
    host = os.environ.get("MASTER_ADDR", "127.0.0.1")
    port = int(os.environ.get("MASTER_PORT", "29500")) + 17
    return TCPStore(host, port, world_size=world, is_master=rank == 0, wait_for_workers=False)


def _visible(local, world):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = vis.split(",")
        return set(ids[:world]) if world > 1 else {ids[local] if local < len(ids) else ids[0]}
    return {str(i) for i in range(world)} if world > 1 else {str(local)}


def _timed(run_step, warmup, steps, barrier, reduce_max, local, world):
    import torch

    for _ in range(warmup):
        run_step()
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler()
    if local == 0:
        sampler.start()
        time.sleep(0.5)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    start.record()
    t0 = time.perf_counter()
    for _ in range(steps):
        run_step()
    end.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop(_visible(local, world)) if local == 0 else None
    device_s = start.elapsed_time(end) / 1000.0
    return reduce_max(device_s), reduce_max(wall), clocks


def _tp_comm(tp):
    from resihp.parallel import fused

    if tp == 1:
        return "none"
    return "fused-nvlink" if fused.ENABLED and tp <= fused.MAX_DEGREE else "nccl"


def _trace_step(step, directory, rank, barrier):
    """One profiled step after the measurement: Chrome trace + top kernels by device time."""
    import json as _json

    import torch
    from torch.profiler import ProfilerActivity, profile

    os.makedirs(directory, exist_ok=True)
    barrier()
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    barrier()
    prof.export_chrome_trace(os.path.join(directory, f"trace_rank{rank}.json"))
    rows = []
    for ev in prof.key_averages():
        device_us = getattr(ev, "device_time_total", 0.0) or getattr(ev, "cuda_time_total", 0.0)
        if device_us > 0:
            rows.append({"name": ev.key[:120], "calls": ev.count, "device_us": round(device_us, 1)})
    rows.sort(key=lambda r: -r["device_us"])
    from resihp.utils.trace import categorize

    with open(os.path.join(directory, f"kernels_rank{rank}.json"), "w") as f:
        _json.dump({"categories": categorize(rows), "top_kernels": rows[:60]}, f, indent=1)


def bench_config(which: int, world: int, iterations: int, layout: tuple[int, int, int] | None = None):
    """The training config the bench runs: BASELINE config ``which`` on ``world`` GPUs
    (in ``layout`` = ``(tp, pp, dp)`` when given, else the config's layout for them)."""
    from resihp.config import TrainConfig

    spec = CONFIGS[which]
    tp, pp, dp = layout if layout is not None else spec["layouts"][world]
    if tp * pp * dp != world:
        raise SystemExit(f"layout tp{tp} pp{pp} dp{dp} does not use {world} GPUs")
    extra = dict(num_kv_heads=None)
    extra.update(spec["extra"])
    return TrainConfig(
        **spec["model"], **extra, batch_size=spec["global_batch"], micro_batch_size=spec["micro_batch"], seed=1,
        tp=tp, pp=pp, dp=dp, iterations=iterations, arch="llama", dtype="bf16",
        sequence_parallel=tp > 1, init_std=0.02, lr=3e-4, beta1=0.9, beta2=0.95, weight_decay=0.1,
        memory_budget_bytes=180 * 10**9,
    )


def _memory(run, plan, config, device):
    """``(measured peak bytes, the planner's estimate)`` for this rank's stage."""
    import torch

    from resihp.memory import estimate_memory
    from resihp.planner.pp import peak_in_flight
    from resihp.recovery import stage_of

    if run is None:
        return 0.0, 0.0
    st = run.stage
    used = torch.cuda.max_memory_allocated(device)
    if st.flat.region is not None:
        used += st.flat.region.numel()
    if st.ws is not None:
        used += st.ws.total
    sp = stage_of(plan, run.rank)
    stages = sorted({s.stage_id for s in plan.stages if s.replica_id == sp.replica_id})
    micro = len(run.runtime.micro_batches)
    est = estimate_memory(config, tp_degree=sp.tp_degree, stage_layers=sp.stage_layers, micro_batches=micro,
                          sequence_length=config.seq_len, vocab_size=config.vocab_size,
                          in_flight_micro_batches=peak_in_flight(micro, stage_index=stages.index(sp.stage_id),
                                                                 num_stages=len(stages)))
    return float(used), float(est.total)


def run_ours(args):
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from resihp.control import ControlPlane
    from resihp.ops import _ext, check_device_errors
    from resihp.plan import build_plan
    from resihp.recovery import initial_run

    rank, world, local = _env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    spec = CONFIGS[args.config]
    layout = tuple(int(x) for x in args.layout.split(",")) if args.layout else None
    if layout is None and world not in spec["layouts"]:
        raise SystemExit(f"config {args.config} runs on {sorted(spec['layouts'])} GPUs, not {world}")
    tp, pp, dp = layout if layout is not None else spec["layouts"][world]
    global_batch, micro_batch = spec["global_batch"], spec["micro_batch"]
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    config = bench_config(args.config, world, args.warmup + args.steps, layout)
    cp = ControlPlane(rank, range(world), _store(rank, world), "nccl", device=device)
    cp.form_world(range(world), epoch=0)
    plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    groups = cp.build_training_groups(plan)
    run = initial_run(plan, rank=rank, groups=groups, device=device, pin=True)
    h2d_bytes = 0
    d2h_bytes = 0
    if run is not None:
        mbs = len(run.runtime.micro_batches)
        if run.stage.is_first or run.stage.is_last:
            h2d_bytes = mbs * micro_batch * config.seq_len * 8
        d2h_bytes = 4 if run.stage.is_last else 0

    def step():
        return run.step() if run is not None else None

    def barrier():
        dist.barrier(group=cp.world_group)

    def reduce_max(x):
        t = torch.tensor([float(x)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=cp.world_group)
        return float(t.item())

    counter = _ext.launch_counter()
    torch.cuda.reset_peak_memory_stats(device)
    for _ in range(args.warmup):
        step()
    counter.launches = 0
    counter.enabled = True
    device_s, wall_s, clocks = _timed(step, 0, args.steps, barrier, reduce_max, local, world)
    counter.enabled = False
    launches = int(reduce_max(counter.launches))
    check_device_errors(local)
    if args.trace:
        _trace_step(step, args.trace, rank, barrier)
    try:
        used, estimate = _memory(run, plan, config, device)
    except Exception as error:  # an auxiliary report must not cost the measurement
        print(f"memory report unavailable: {error}", file=sys.stderr)
        used, estimate = 0.0, 0.0
    mem = torch.tensor([used, estimate])
    dist.all_reduce(mem, op=dist.ReduceOp.MAX, group=cp.world_group)
    bytes_in = torch.tensor([float(h2d_bytes), float(d2h_bytes)])
    dist.all_reduce(bytes_in, group=cp.world_group)
    tokens = args.steps * global_batch * config.seq_len
    value = tokens / device_s
    e2e = tokens / wall_s
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * device_s / args.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded uniform tokens), random-init weights",
            "config": {"model": spec["name"], "baseline_config": args.config, "global_batch": global_batch,
                       "micro_batch": micro_batch, "seq_len": config.seq_len,
                       "parallelism": f"tp{tp}-pp{pp}-dp{dp}" + ("-sp" if tp > 1 else ""),
                       "tp_comm": _tp_comm(tp),
                       "dp_comm": ("fused-nvlink+adamw" if os.environ.get("RESIHP_FUSED_DP", "1") != "0" else "nccl") if dp > 1 else "none",
                       "l2": "inputs larger than L2 (weights/activations >> 126 MB)"},
            "clocks": clocks,
            "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": int(bytes_in[0]),
                    "d2h_bytes_per_step": int(bytes_in[1])},
            "gpu_launches": launches,
            "memory": {"peak_gib": round(float(mem[0]) / 2**30, 2), "planner_estimate_gib": round(float(mem[1]) / 2**30, 2),
                       "note": "max over ranks; peak = caching-allocator peak + flat-state region + TP workspace"},
            "impl": "resihp",
        }
        print(json.dumps(line), flush=True)
    if run is not None:
        run.stage.close_comm()
    del run
    cp.destroy_training_groups()
    dist.barrier(group=cp.world_group)
    dist.destroy_process_group()


def run_reference(args):
    if args.config != 2:
        print(json.dumps({"impl": "reference", "unavailable": f"config {args.config} needs GQA / sequence parallelism "
                          "/ recompute / bf16, which the reference cannot express"}))
        return
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "resihp")):
        print(json.dumps({"impl": "reference", "unavailable": "reference not installed under baseline/_ref"}))
        return
    sys.path = [ref] + [p for p in sys.path if os.path.abspath(p or ".") != ROOT]
    import torch
    import torch.distributed as dist

    import resihp
    assert os.path.abspath(resihp.__file__).startswith(ref), resihp.__file__
    from resihp.config import TrainConfig
    from resihp.control import ControlPlane
    from resihp.plan import build_plan
    from resihp.recovery import initial_run

    rank, world, local = _env()
    tp, pp, dp = LAYOUTS[world]
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    config = TrainConfig(model_dim=MODEL["model_dim"], num_layers=MODEL["num_layers"], num_heads=MODEL["num_heads"],
                         batch_size=GLOBAL_BATCH, micro_batch_size=MICRO_BATCH, seed=1, tp=tp, pp=pp, dp=dp,
                         iterations=args.warmup + args.steps)
    cp = ControlPlane(rank, range(world), _store(rank, world), "nccl", vocab_size=MODEL["vocab_size"],
                      sequence_length=MODEL["seq_len"])
    cp.form_world(range(world), epoch=0)
    plan = build_plan(config, step=0, version=0, vocab_size=MODEL["vocab_size"], sequence_length=MODEL["seq_len"])
    cp.build_training_groups(plan)
    run = initial_run(plan, rank=rank, vocab_size=MODEL["vocab_size"], sequence_length=MODEL["seq_len"],
                      tp_group=cp.tp_group, executor_group=cp.executor_group, boundary_groups=cp.boundary_groups,
                      device=device)

    def step():
        return run.step() if run is not None else None

    def barrier():
        dist.barrier(group=cp.world_group)

    def reduce_max(x):
        t = torch.tensor([float(x)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=cp.world_group)
        return float(t.item())

    device_s, wall_s, clocks = _timed(step, args.warmup, args.steps, barrier, reduce_max, local, world)
    tokens = args.steps * GLOBAL_BATCH * MODEL["seq_len"]
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(tokens / device_s, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * device_s / args.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded uniform tokens), random-init weights",
            "config": {"model": "gpt2-arch 1.3b (24L, d2048, 16H, FFN 4d, V32000): closest reference shape",
                       "global_batch": GLOBAL_BATCH, "micro_batch": MICRO_BATCH, "seq_len": MODEL["seq_len"],
                       "parallelism": f"tp{tp}-pp{pp}-dp{dp}", "l2": "inputs larger than L2"},
            "clocks": clocks,
            "e2e": {"value": round(tokens / wall_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": None,
                    "d2h_bytes_per_step": None},
            "impl": "reference",
        }), flush=True)
    cp.shutdown()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
