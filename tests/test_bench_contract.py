"""The host-side parts of ``bench.py`` that decide what a reported number means.

* Every (config, GPU count) the bench accepts plans to exactly the layout its JSON line
  names in ``parallelism`` -- a planner change that picked another TP degree or stage
  count would otherwise silently change the measured configuration.
* The clock summary keeps only the visible GPUs' samples and names every throttle reason
  that was active.
* The memory report reads the attributes it needs from a real run (here a CPU/Gloo TP2
  run) and matches the planner's estimate for that stage.
"""

import json
import os
from pathlib import Path

import pytest

import bench
from harness import read_results, run_ranks, write_result
from resihp.memory import estimate_memory
from resihp.planner.pp import peak_in_flight
from resihp.plan import build_plan


@pytest.mark.parametrize("which", sorted(bench.CONFIGS))
def test_every_bench_layout_plans_as_reported(which):
    for world, (tp, pp, dp) in bench.CONFIGS[which]["layouts"].items():
        config = bench.bench_config(which, world, 8)
        plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
        assert tuple(plan.active_ranks) == tuple(range(world))
        assert {s.tp_degree for s in plan.stages} == {tp}, (which, world)
        assert len({s.replica_id for s in plan.stages}) == dp
        assert len(plan.stages) == pp * dp
        assert config.sequence_parallel == (tp > 1) and config.dtype == "bf16"


def test_parse_defaults_fit_the_timing_rules(monkeypatch):
    monkeypatch.setattr("sys.argv", ["bench.py"])
    args = bench.parse()
    assert args.gpus == 1 and args.warmup >= 3 and args.steps >= 1 and args.impl == "resihp" and args.config == 2


def test_clock_summary_filters_gpus_and_names_reasons():
    sampler = bench.ClockSampler()
    row = lambda gpu, mhz, cap: [gpu, str(mhz), "1965", "900.0", "0x4", "Not Active", "Not Active", "Not Active", cap]
    sampler.rows = [row("0", 1800, "Active"), row("0", 1900, "Not Active"), row("0", 1700, "Not Active"),
                    row("1", 500, "Not Active"), row("0", "[N/A]", "Not Active")]
    out = sampler.stop({"0"})
    assert out["sm_mhz"] == 1800.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"] and out["samples"] == 4
    assert bench.ClockSampler().stop({"0"})["reasons"] == ["unsampled"]


def test_visible_devices(monkeypatch):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3,5")
    assert bench._visible(1, 1) == {"5"} and bench._visible(0, 2) == {"3", "5"}
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES")
    assert bench._visible(2, 1) == {"2"} and bench._visible(0, 4) == {"0", "1", "2", "3"}


CONFIG = dict(model_dim=32, num_layers=2, num_heads=4, batch_size=4, micro_batch_size=2, seed=2, tp=2, pp=1, dp=1,
              iterations=2, arch="llama", vocab_size=32, seq_len=8, ffn_dim=64)


def _memory_entry(rank, env, out_dir):
    os.environ.update(env)
    import torch

    torch.set_num_threads(1)
    torch.cuda.max_memory_allocated = lambda device=None: 1000  # the caching allocator's peak on a GPU
    from resihp.config import TrainConfig
    from resihp.control import ControlPlane
    from resihp.recovery import initial_run

    config = TrainConfig(**CONFIG)
    cp = ControlPlane.initialize(training_backend="gloo")
    plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len)
    groups = cp.build_training_groups(plan)
    run = initial_run(plan, rank=rank, groups=groups)
    run.step()
    used, estimate = bench._memory(run, plan, config, "cpu")
    write_result(out_dir, rank, {"used": used, "estimate": estimate, "micro": len(run.runtime.micro_batches)})
    cp.shutdown()


@pytest.mark.slow
def test_memory_report_reads_a_real_run(tmp_path):
    codes = run_ranks(_memory_entry, 2, str(tmp_path))
    assert set(codes.values()) == {0}, codes
    results = read_results(tmp_path, [0, 1])
    from resihp.config import TrainConfig

    config = TrainConfig(**CONFIG)
    for r in results.values():
        want = estimate_memory(config, tp_degree=2, stage_layers=2, micro_batches=r["micro"], sequence_length=8,
                               vocab_size=32, in_flight_micro_batches=peak_in_flight(r["micro"], stage_index=0,
                                                                                     num_stages=1)).total
        assert r["estimate"] == float(want) and r["used"] >= 1000
    assert json.loads(Path(tmp_path, "result_0.json").read_text())["micro"] == 2


def test_every_gpu_shape_we_run_passes_the_kernel_shape_rules():
    """The set-up check of the bf16 kernels' shape rules accepts every shape the bench,
    the recovery bench, the smoke run and the GPU tests run (at each TP degree they use
    or a fail-stop can leave), and names the rule a bad shape breaks."""
    import bench_recovery
    from resihp.config import TrainConfig
    from resihp.models.layout import kernel_shape_problems

    for which, spec in bench.CONFIGS.items():
        for world, (tp, _pp, _dp) in spec["layouts"].items():
            config = bench.bench_config(which, world, 8)
            for degree in sorted({1, tp}):
                assert kernel_shape_problems(config, degree) == [], (which, world, degree)
    base = dict(batch_size=64, micro_batch_size=2, seed=1, tp=2, pp=2, dp=2, iterations=1, arch="llama", dtype="bf16")
    recovery = [dict(bench_recovery.MODEL), dict(bench_recovery.MODEL, num_layers=4, model_dim=1024, num_heads=8,
                                                  ffn_dim=2752, seq_len=1024)]
    gpu_tests = [dict(model_dim=256, num_layers=2, num_heads=h, vocab_size=1024, seq_len=256, ffn_dim=512)
                 for h in (2, 4)]
    for shape in recovery + gpu_tests:
        for degree in (1, 2):
            assert kernel_shape_problems(TrainConfig(**base, **shape), degree) == [], (shape, degree)
    bad = TrainConfig(**base, num_layers=2, model_dim=96, num_heads=4, vocab_size=1001, seq_len=100, ffn_dim=100)
    problems = " | ".join(kernel_shape_problems(bad, 2))
    for rule in ("head_dim 24", "seq_len 100", "model_dim 96", "vocabulary shard 500", "FFN shard 50"):
        assert rule in problems, (rule, problems)


def test_recovery_bench_reads_interleaved_reference_output():
    """The reference's ranks share stdout without line-atomic writes: JSON objects can run
    together or be split by other text; every whole object is still recovered, in order."""
    import bench_recovery

    text = ('noise {"refstep": {"rank": 0, "step_s": 0.1}}{"refrecovery": {"rank": 2, "event": 2, "seconds": 1.5}}\n'
            'W1202 warning {"launch": {"killed_ranks": [1]}} {broken\n{"step": 3, "loss": 2.0}')
    objs = bench_recovery._json_objects(text)
    assert [list(o)[0] for o in objs] == ["refstep", "refrecovery", "launch", "step"]
    assert objs[1]["refrecovery"]["event"] == 2


def test_layout_override_plans_as_asked():
    for world, layout in ((2, (1, 1, 2)), (4, (1, 1, 4)), (4, (2, 1, 2)), (8, (1, 1, 8))):
        config = bench.bench_config(2, world, 8, layout)
        plan = build_plan(config, step=0, version=0, vocab_size=config.vocab_size, sequence_length=config.seq_len,
                          memory_budget=config.memory_budget_bytes)
        assert {s.tp_degree for s in plan.stages} == {layout[0]} and len(plan.stages) == layout[1] * layout[2]
        assert config.sequence_parallel == (layout[0] > 1)
    with pytest.raises(SystemExit, match="does not use 4 GPUs"):
        bench.bench_config(2, 4, 8, (2, 1, 1))
