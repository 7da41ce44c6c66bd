"""The two Principle A acceptance contracts (reference: ``resihp/verify.py:63-299``).

**A1 -- before resume.** Once reconfiguration is done, this rank's complete state --
``param``, ``exp_avg``, ``exp_avg_sq``, ``step`` -- equals the pre-failure checkpoint,
sliced by the new plan's layout, under ``torch.equal``. Recovery moves bytes; it does
not compute.

**A2 -- after resume.** The resumed run is compared against a single-process oracle
started from the same checkpoint and stepped on the same batches
(:func:`steps_from_anchor`), never against an uninterrupted run from step 0. Gradients
must sit in the reassociation band (``rtol=1e-4``, ``atol=1e-5``); parameters get the
AdamW-conditioned allowance ``atol + rtol |p| + 2 lr |dg| / denom``: where
``sqrt(v_hat)`` has decayed towards ``eps`` the update degenerates to ``lr * sign(g)``,
so a reassociation-sized gradient difference can move a parameter by up to ``2 lr``.
"""

from __future__ import annotations

import math

import torch

from .checkpoint import load_anchor
from .parallel.tp import local_slice
from .recovery import checkpoint_mismatches, stage_layout, stage_of
from .reference import ReferenceRun

RTOL = 1e-4
ATOL = 1e-5


# --- A1 --------------------------------------------------------------------------------


def matches_checkpoint(run, plan, rank, checkpoint_path) -> bool:
    anchor, _ = load_anchor(checkpoint_path)
    return not checkpoint_mismatches(run, plan=plan, rank=rank, anchor=anchor)


def assert_equals_checkpoint(run, *, plan, rank, checkpoint_path) -> None:
    anchor, _ = load_anchor(checkpoint_path)
    problems = checkpoint_mismatches(run, plan=plan, rank=rank, anchor=anchor)
    if problems:
        raise AssertionError(f"rank {rank} does not equal the checkpoint under plan v{plan.version}: {problems}")


def checkpoint_mismatches_at(run, *, plan, rank, checkpoint_path) -> list[str]:
    """Every way this rank's state differs from the checkpoint at ``checkpoint_path``."""
    anchor, _ = load_anchor(checkpoint_path)
    return checkpoint_mismatches(run, plan=plan, rank=rank, anchor=anchor)


# --- A2 --------------------------------------------------------------------------------


def _check_constants(config, vocab_size, sequence_length):
    """The reference passes its run constants alongside the config; here the config
    carries them, and any value passed must agree."""
    for name, given, have in (("vocab_size", vocab_size, config.vocab_size),
                              ("sequence_length", sequence_length, config.seq_len)):
        if given is not None and given != have:
            raise ValueError(f"{name}={given} does not match the config ({have})")


def batch(config, index, *, device, vocab_size=None, sequence_length=None):
    """Iteration ``index``'s fixed token batch -- the same stream a run consumes."""
    from .reference import token_stream

    _check_constants(config, vocab_size, sequence_length)
    return token_stream(config)[index].to(device)


def denominator(config, exp_avg_sq=None, step=None):
    """AdamW's ``sqrt(v / bias_correction2) + eps`` after its ``step``-th update.

    ``denominator(config, exp_avg_sq, step)``; or, as the reference calls it,
    ``denominator(state)`` with ``state = {"exp_avg_sq", "step"}`` and the default
    AdamW hyper-parameters.
    """
    if exp_avg_sq is None:
        from .config import TrainConfig

        state, defaults = config, TrainConfig.__dataclass_fields__
        exp_avg_sq, step = state["exp_avg_sq"], state["step"]
        beta2, eps = defaults["beta2"].default, defaults["adam_eps"].default
    else:
        beta2, eps = config.beta2, config.adam_eps
    bc2 = 1 - beta2 ** float(step)
    return exp_avg_sq.sqrt() / math.sqrt(bc2) + eps



def reference_steps(config, *, count, device="cpu", vocab_size=None, sequence_length=None) -> list[dict]:
    """The no-failure oracle: ``count`` full-batch steps from the seeded initialisation."""
    _check_constants(config, vocab_size, sequence_length)
    run = ReferenceRun(config, device=device)
    return [step_record(run) for _ in range(count)]


def step_record(run, optimizer=None, tokens=None, *, vocab_size=None) -> dict:
    """One full-batch oracle step: its gradients, new parameters, moments and denominators.

    ``step_record(run)`` steps a :class:`~resihp.reference.ReferenceRun`. The reference's
    form ``step_record(model, optimizer, tokens, vocab_size=V)`` steps a module-form model
    (:class:`resihp.model.ReferenceTransformer`) with its ``torch.optim.AdamW`` and
    returns the reference's keys: loss, grads, params, moments.
    """
    if optimizer is not None:
        return _module_step_record(run, optimizer, tokens, vocab_size)
    stage = run.stage
    tokens = run.batches[run.cursor].to(run.device)
    stage.zero_grad()
    b, s = tokens.shape
    loss = stage.forward(tokens=tokens, loss_scale=1.0 / (b * (s - 1)))
    loss.backward()
    grads = {n: stage.g[n].detach().clone() for n in stage.logical_state_dict()}
    stage.optimizer_step()
    run.cursor += 1
    params, denoms = {}, {}
    for n, (view, _d) in stage.local_shards().items():
        params[n] = view.detach().clone()
        denoms[n] = denominator(stage.config, stage.moment_views(n)["exp_avg_sq"], stage.flat.step)
    return {"loss": float(loss.detach()), "grads": grads, "params": params, "denoms": denoms}


def _module_step_record(model, optimizer, tokens, vocab_size) -> dict:
    from .reference import next_token_loss

    loss = next_token_loss(model(tokens), tokens, vocab_size)
    optimizer.zero_grad()
    loss.backward()
    named = model.logical_state_dict()
    grads = {n: p.grad.detach().clone() for n, p in named.items()}
    optimizer.step()
    return {
        "loss": float(loss.detach()), "grads": grads,
        "params": {n: p.detach().clone() for n, p in named.items()},
        "moments": {n: {k: optimizer.state[p][k].detach().clone() for k in ("exp_avg", "exp_avg_sq", "step")}
                    for n, p in named.items()},
    }


def steps_from_anchor(config, anchor, *, start: int, count: int, device="cpu", vocab_size=None,
                      sequence_length=None) -> list[dict]:
    """A2's oracle: ``count`` full-batch steps from the checkpoint ``anchor`` at cursor ``start``."""
    _check_constants(config, vocab_size, sequence_length)
    full = {n: e["param"] for n, e in anchor.items()}
    moments = {n: e for n, e in anchor.items() if "exp_avg" in e}
    run = ReferenceRun(config, device=device, full_state=full, moments=moments, cursor=start)
    return [step_record(run) for _ in range(count)]


def compare_shards(stage, record, *, lr: float) -> dict:
    """Measure one stage's shards against an oracle record (JSON-serialisable summary)."""
    grad_close = step_close = True
    max_grad = max_param = 0.0
    worst = None
    for name, (param, dim) in stage.local_shards().items():
        sliced = (dim, stage.tp_rank, stage.tp_size)
        want_p = local_slice(record["params"][name], *sliced).to(param.device)
        want_g = local_slice(record["grads"][name], *sliced).to(param.device)
        denom = local_slice(record["denoms"][name], *sliced).to(param.device)
        got_g = stage.g[name]
        dg = (got_g - want_g).abs()
        dp = (param.detach() - want_p).abs()
        allowed = ATOL + RTOL * want_p.abs() + 2 * lr * dg / denom
        grad_close &= bool(torch.allclose(got_g, want_g, rtol=RTOL, atol=ATOL))
        ok = bool((dp <= allowed).all())
        step_close &= ok
        max_grad = max(max_grad, dg.max().item())
        max_param = max(max_param, dp.max().item())
        if not ok and worst is None:
            worst = {"name": name, "excess": (dp - allowed).max().item()}
    return {"grad_close": grad_close, "step_close": step_close, "max_grad_diff": max_grad,
            "max_param_diff": max_param, "worst_param": worst, "tp_size": stage.tp_size}


def assert_matches_reference(comparison: dict, *, label: str = "") -> None:
    where = f"{label}: " if label else ""
    if not comparison["grad_close"]:
        raise AssertionError(f"{where}gradients left the reassociation band: {comparison}")
    if not comparison["step_close"]:
        raise AssertionError(f"{where}post-AdamW parameters differ beyond AdamW's own conditioning: {comparison}")


__all__ = [
    "RTOL", "ATOL", "matches_checkpoint", "assert_equals_checkpoint", "checkpoint_mismatches_at", "batch",
    "denominator", "step_record", "reference_steps", "steps_from_anchor", "compare_shards",
    "assert_matches_reference", "stage_of", "stage_layout",
]
