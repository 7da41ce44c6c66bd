#!/usr/bin/env python
"""Fail-stop recovery benchmark: recovery seconds and tokens/s around kills.

Runs the real launcher (``python -m resihp.launch``) on the config-2 model -- Llama-style
1.3B, bf16 with FP32 master weights and AdamW, TP2 x PP2 x DP2 on 8 GPUs, sequence 2048,
micro-batch 2, global batch 64, synthetic seeded tokens -- with a failure schedule that
SIGKILLs GPU 5 after step 30 and GPU 2 after step 60. Each fail-stop is detected through
the launcher's store, replanned by the memory-aware planner (180 GB budget per GPU),
and the parameters plus AdamW state move to their new owners peer to peer; no checkpoint
is needed because every lost shard survives on a peer replica. (Without a peer replica,
DP = 1, the checkpoint is committed every step, as the reference does.)

Prints one JSON line: per event the recovery time (failure -> end of the first resumed
step, max over surviving ranks) with its phases, and tokens/s of the steps before and
after each event.

    python bench_recovery.py [--gpus 8] [--kills 30:5,60:2] [--iterations 70]
    python bench_recovery.py --config 1     # CPU/Gloo, 4 ranks, kill rank 3 after step 8
    python bench_recovery.py --config 1 --reference-model [--impl reference]
        # config 1's topology and kill on the closest model the reference can run (GPT-2
        # blocks, vocab 1024, seq 128, seed 1), by this framework or by the unmodified
        # reference timed through baseline/recovery_hook
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.abspath(__file__))
MODEL = dict(model_dim=2048, num_layers=24, num_heads=16, ffn_dim=5504, vocab_size=32000, seq_len=2048)
LAYOUTS = {2: (2, 1, 1), 4: (2, 2, 1), 8: (2, 2, 2)}
# BASELINE config 1 (CPU/Gloo, FP32): Llama d256 L4 H4, SwiGLU 688, vocab 1024, tied embeddings,
# seq 128, 4 micro-batches of 2, TP2 x PP2 x DP1, AdamW lr 1e-3 betas (0.9, 0.95) wd 0.1, seed 0.
CONFIG1 = dict(model_dim=256, num_layers=4, num_heads=4, ffn_dim=688, vocab_size=1024, seq_len=128, batch_size=8,
               micro_batch_size=2, seed=0, tp=2, pp=2, dp=1, iterations=20, arch="llama", dtype="fp32",
               tied_embeddings=True, norm_eps=1e-5, rope_theta=10000.0, init_std=0.02, lr=1e-3, beta1=0.9,
               beta2=0.95, weight_decay=0.1)
# The closest run the reference can express: GPT-2 blocks (its only model), FP32, its AdamW
# settings, seed 1 (it rejects seed 0); vocabulary and sequence set through its run
# constants by the timing hook.
REFERENCE_MODEL1 = dict(model_dim=256, num_layers=4, num_heads=4, batch_size=8, micro_batch_size=2, seed=1, tp=2,
                        pp=2, dp=1, iterations=20, memory_budget_bytes=None)


def _json_objects(text):
    """Every JSON object in ``text`` (the reference's ranks share stdout without
    line-atomic writes, so objects can run together on one line)."""
    dec = json.JSONDecoder()
    out, i = [], 0
    while True:
        j = text.find("{", i)
        if j < 0:
            return out
        try:
            obj, i = dec.raw_decode(text, j)
            out.append(obj)
        except json.JSONDecodeError:
            i = j + 1


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=8)
    p.add_argument("--kills", default="30:5,60:2", help="after_iteration:rank,...")
    p.add_argument("--iterations", type=int, default=70)
    p.add_argument("--timeout", type=float, default=1500)
    p.add_argument("--small", action="store_true", help="a 4-layer model (quick check)")
    p.add_argument("--layout", default=None, help="tp,pp,dp (default: config 4's layout for --gpus)")
    p.add_argument("--config", type=int, choices=(1, 4), default=4,
                   help="4: the 1.3B GPU run (default); 1: the CPU/Gloo run of BASELINE config 1")
    p.add_argument("--shipped", action="store_true",
                   help="the shipped configs/train.json + configs/failures.json schedule on CPU/Gloo "
                        "(8 ranks, 5 fail-stops); with --impl reference, the unmodified reference runs it")
    p.add_argument("--reference-model", action="store_true",
                   help="config 1 only: the GPT-2 config-1-like model the reference can express")
    p.add_argument("--impl", choices=("resihp", "reference"), default="resihp",
                   help="config 1 with --reference-model: run the unmodified reference instead")
    p.add_argument("--checkpoint-every", type=int, default=None,
                   help="commit the logical checkpoint every N steps (default: every step without a peer "
                        "replica, never with one)")
    return p.parse_args()


def main():
    args = parse()
    if args.impl == "reference" and not (args.shipped or (args.config == 1 and args.reference_model)):
        raise SystemExit("--impl reference runs --shipped, or config 1 with --reference-model")
    if args.shipped:
        with open(os.path.join(ROOT, "configs", "train.json")) as f:
            config = json.load(f)
        with open(os.path.join(ROOT, "configs", "failures.json")) as f:
            shipped = json.load(f)["events"]
        tp, pp, dp = config["tp"], config["pp"], config["dp"]
        args.gpus = tp * pp * dp
        args.kills = ",".join(f"{e['after_iteration']}:{e['failed_rank']}" for e in shipped)
    elif args.config == 1:
        config = dict(CONFIG1)
        if args.reference_model:
            config = dict(REFERENCE_MODEL1)
        tp, pp, dp = config["tp"], config["pp"], config["dp"]
        args.gpus = tp * pp * dp
        args.kills = "8:3"
    else:
        tp, pp, dp = (tuple(int(x) for x in args.layout.split(",")) if args.layout else LAYOUTS[args.gpus])
        if tp * pp * dp != args.gpus:
            raise SystemExit(f"layout {tp}x{pp}x{dp} does not use {args.gpus} GPUs")
        model = dict(MODEL)
        if args.small:
            model.update(num_layers=4, model_dim=1024, num_heads=8, ffn_dim=2752, seq_len=1024)
        config = dict(
            **model, batch_size=64, micro_batch_size=2, seed=1, tp=tp, pp=pp, dp=dp, iterations=args.iterations,
            arch="llama", dtype="bf16", sequence_parallel=True, init_std=0.02, lr=3e-4, beta1=0.9, beta2=0.95,
            weight_decay=0.1, memory_budget_bytes=180 * 10**9,
            checkpoint_every=args.checkpoint_every or (1 if dp == 1 else 1_000_000),
        )
    kills = [tuple(int(x) for x in k.split(":")) for k in args.kills.split(",") if k]
    failures = {"events": [{"after_iteration": a, "failed_rank": r} for a, r in kills]}
    with tempfile.TemporaryDirectory() as tmp:
        cfg_path = os.path.join(tmp, "train.json")
        fail_path = os.path.join(tmp, "failures.json")
        with open(cfg_path, "w") as f:
            json.dump(config, f)
        with open(fail_path, "w") as f:
            json.dump(failures, f)
        env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0", RESIHP_CHECKPOINT=os.path.join(tmp, "ck.pt"))
        if args.config == 1 or args.shipped:
            env.update(CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")  # the CPU/Gloo runs
        if args.impl == "reference":
            ref = os.path.join(ROOT, "baseline", "_ref")
            if not os.path.isdir(os.path.join(ref, "resihp")):
                raise SystemExit("reference not installed under baseline/_ref")
            env.update(PYTHONPATH=os.pathsep.join([os.path.join(ROOT, "baseline", "recovery_hook"), ref]),
                       RESIHP_REFHOOK="1")
            if not args.shipped:  # config 1's token-stream shape; the shipped config uses the defaults
                env.update(RESIHP_REF_VOCAB="1024", RESIHP_REF_SEQ="128")
        elif args.reference_model:
            with open(cfg_path, "w") as f:
                json.dump(dict(config, vocab_size=1024, seq_len=128), f)
        env.setdefault("RESIHP_GROUP_TIMEOUT", "120")
        out = subprocess.run(
            [sys.executable, "-m", "resihp.launch", "--config", cfg_path, "--failures", fail_path,
             "--timeout", str(args.timeout)],
            cwd=tmp, env=env, capture_output=True, text=True, timeout=args.timeout + 120,
        )
    lines = _json_objects(out.stdout)
    if args.impl == "reference":
        for l in lines:
            if "refrecovery" in l:
                rec = l.pop("refrecovery")
                event = rec.get("event", 1)
                l["recovery"] = dict(rec, after_iteration=kills[event - 1][0], phases={}, plan_version=event)
            if "refstep" in l:
                l["step"], l["step_s"] = -1, l.pop("refstep")["step_s"]
    launch = next((l["launch"] for l in lines if "launch" in l), None)
    steps: dict[int, list] = {}
    for l in lines:
        if "step" in l:
            steps.setdefault(l["step"], []).append(l["step_s"])
    seq_len = config.get("seq_len", 128 if args.reference_model else 16)
    tokens = config["batch_size"] * seq_len
    if args.shipped:
        label = "shipped configs/train.json (gpt2, CPU/Gloo, FP32)"
    elif args.config == 1:
        label = ("gpt2 config-1-like (CPU/Gloo, FP32)" if args.reference_model else "llama-config1 (CPU/Gloo, FP32)")
    else:
        label = "llama-1.3b" if not args.small else "llama-small"
    all_steps = sorted(x for v in steps.values() for x in v)
    step_rate = {it: tokens / max(v) for it, v in steps.items()}
    events = []
    for a, r in kills:
        rec = [l["recovery"] for l in lines if "recovery" in l and l["recovery"]["after_iteration"] == a]
        if not rec:
            events.append({"after_iteration": a, "failed_rank": r, "recovered": False})
            continue
        worst = max(rec, key=lambda x: x["seconds"])
        before = [step_rate[i] for i in range(max(2, a - 5), a + 1) if i in step_rate]
        after = [step_rate[i] for i in range(a + 2, a + 8) if i in step_rate]
        events.append({
            "after_iteration": a, "failed_rank": r, "recovered": True,
            "recovery_s": round(worst["seconds"], 3), "safe_point_s": round(worst["safe_point_s"], 3),
            "first_resumed_step_s": round(worst.get("first_step_s", 0.0), 3),
            "phases_s": {k: round(v, 3) for k, v in worst["phases"].items()},
            "plan_version": worst["plan_version"],
            "tokens_per_s_before": round(statistics.median(before), 1) if before else None,
            "tokens_per_s_after": round(statistics.median(after), 1) if after else None,
        })
    print(json.dumps({
        "metric": "fail-stop recovery seconds (failure -> end of first resumed step, max over survivors)",
        "impl": args.impl, "median_step_s": round(statistics.median(all_steps), 4) if all_steps else None,
        "n_gpus": 0 if (args.config == 1 or args.shipped) else args.gpus, "ranks": args.gpus,
        "config": {"model": label, "baseline_config": None if args.shipped else args.config,
                   "parallelism": f"tp{tp}-pp{pp}-dp{dp}" + ("-sp" if config.get("sequence_parallel") else ""),
                   "dtype": config.get("dtype", "fp32"), "global_batch": config["batch_size"], "seq_len": seq_len},
        "events": events, "launch": launch, "launcher_rc": out.returncode,
        "stopped": [l for l in lines if "stopped" in l],
        "steps_seen": sorted(steps),
        "recovery_lines": [l["recovery"] for l in lines if "recovery" in l][:4 * len(kills)],
        "stderr_tail": out.stderr[-1500:] if out.returncode else "",
    }), flush=True)


if __name__ == "__main__":
    main()
