"""Deterministic random planning scenarios shared by the differential planner test.

Each scenario is plain JSON (config fields, planning inputs, a failure sequence) so the
same scenario can be replayed by this framework's planner and, in a subprocess, by the
reference implementation installed under ``baseline/_ref``.
"""

import random


def scenarios(count: int, seed: int = 7):
    rng = random.Random(seed)
    out = []
    while len(out) < count:
        tp = rng.choice([1, 2, 4])
        pp = rng.choice([1, 2, 3])
        dp = rng.choice([1, 2, 3])
        heads = rng.choice([2, 4, 8])
        dim = heads * rng.choice([4, 8, 16])
        layers = rng.randint(pp, pp + 5)
        micro = rng.choice([1, 2])
        batch = micro * rng.randint(1, 6)
        vocab = rng.choice([None, 32, 48, 64])
        seq = rng.choice([1, 8])
        budget = None
        if vocab is not None and rng.random() < 0.4:
            budget = rng.randint(20_000, 400_000)
        world = tp * pp * dp
        victims = list(range(world))
        rng.shuffle(victims)
        fails = victims[: rng.randint(1, max(1, world - 1))]
        out.append(
            {
                "config": dict(
                    model_dim=dim, num_layers=layers, num_heads=heads, batch_size=batch,
                    micro_batch_size=micro, seed=1, tp=tp, pp=pp, dp=dp, iterations=4,
                    memory_budget_bytes=budget,
                ),
                "vocab": vocab,
                "seq": seq,
                "budget": budget,
                "failures": fails,
            }
        )
    return out


def replay(module_config, module_plan, scenario):
    """Run one scenario: initial plan, then one replan per failure; digests or stop codes."""
    config = module_config.TrainConfig(**scenario["config"])
    kwargs = dict(memory_budget=scenario["budget"], sequence_length=scenario["seq"], vocab_size=scenario["vocab"])
    trace = []
    try:
        plan = module_plan.build_plan(config, step=0, version=0, **kwargs)
    except module_plan.InfeasiblePlan as error:
        return [["stop", error.reason.code]]
    trace.append(["plan", plan.digest])
    failed = []
    for i, rank in enumerate(scenario["failures"]):
        failed.append(rank)
        try:
            plan = module_plan.build_plan(
                config, step=i + 1, version=plan.version + 1, failed_ranks=failed, previous=plan, **kwargs
            )
        except module_plan.InfeasiblePlan as error:
            trace.append(["stop", error.reason.code])
            break
        trace.append(["plan", plan.digest])
    return trace
