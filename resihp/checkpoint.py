"""The atomic, topology-free logical checkpoint.

Format (identical keys and digest to the reference, ``resihp/checkpoint.py:64-108``, so
either implementation reads the other's files)::

    {"format_version": 1, "completed_steps": int, "plan_version": int,
     "identity": {...shape- and data-defining config fields...},
     "params": {name: full FP32 tensor},
     "optim":  {name: {"exp_avg", "exp_avg_sq", "step"}},
     "cpu_rng_state": ByteTensor, "cuda_rng_state": [ByteTensor] | None,
     "digest": sha256 over the scalar fields and every tensor's dtype, shape and bytes}

``identity`` holds the reference's fields for GPT-2 blocks and adds the Llama shape
fields otherwise; topology (TP/PP/DP, micro-batch size) is deliberately absent.
Writes go to ``<path>.tmp``, are read back and compared with memory, then ``os.replace``-d
over the single canonical path; any failure removes the temp file and leaves the last
valid checkpoint untouched. Every problem a load can find is reported as its own
:class:`CheckpointError` (missing file, unreadable payload, format, identity, names,
shapes, cursor/step consistency, digest -- digest last).
"""

from __future__ import annotations

from hashlib import sha256
import json
import os
from pathlib import Path

import torch

from .config import TrainConfig

FORMAT_VERSION = 1
OPTIM_STATES = ("exp_avg", "exp_avg_sq", "step")


class CheckpointError(RuntimeError):
    """A checkpoint is missing, unreadable, inconsistent or corrupted."""


def identity(config: TrainConfig) -> dict:
    out = {
        "model_dim": config.model_dim,
        "num_layers": config.num_layers,
        "num_heads": config.num_heads,
        "batch_size": config.batch_size,
        "seed": config.seed,
        "vocab_size": config.vocab_size,
        "sequence_length": config.seq_len,
    }
    if config.arch != "gpt2":
        out.update(
            arch=config.arch, ffn_dim=config.ffn, num_kv_heads=config.kv_heads,
            tied_embeddings=config.tied_embeddings,
        )
    return out


def payload_digest(payload: dict) -> str:
    h = sha256()
    scalars = {k: payload[k] for k in ("format_version", "completed_steps", "plan_version", "identity")}
    h.update(json.dumps(scalars, sort_keys=True).encode("utf-8"))

    def add(t):
        arr = t.detach().cpu().contiguous().numpy()
        h.update(repr(arr.dtype).encode("utf-8"))
        h.update(repr(arr.shape).encode("utf-8"))
        h.update(arr.tobytes())

    for name in sorted(payload["params"]):
        h.update(name.encode("utf-8"))
        add(payload["params"][name])
    for name in sorted(payload["optim"]):
        for key in OPTIM_STATES:
            value = payload["optim"][name][key]
            h.update(f"{name}:{key}".encode("utf-8"))
            add(value if torch.is_tensor(value) else torch.tensor(value))
    add(payload["cpu_rng_state"])
    cuda = payload["cuda_rng_state"]
    h.update(b"cuda:none" if cuda is None else b"cuda")
    for t in cuda or ():
        add(t)
    return h.hexdigest()


def rng_states() -> tuple:
    """``(cpu, cuda or None)`` generator states, as the payload stores them."""
    return torch.get_rng_state(), (torch.cuda.get_rng_state_all() if torch.cuda.is_available() else None)


def build_payload(config: TrainConfig, full: dict, *, completed_steps: int, plan_version: int,
                  rng: tuple | None = None) -> dict:
    """Payload from a full logical state ``{name: {param[, exp_avg, exp_avg_sq, step]}}``.

    ``rng`` are the generator states to record (default: the current ones).
    """
    cpu_rng, cuda_rng = rng if rng is not None else rng_states()
    params = {n: f["param"].detach().to("cpu", torch.float32).clone() for n, f in full.items()}
    optim = {}
    for n, f in full.items():
        if "exp_avg" in f:
            optim[n] = {
                "exp_avg": f["exp_avg"].detach().to("cpu", torch.float32).clone(),
                "exp_avg_sq": f["exp_avg_sq"].detach().to("cpu", torch.float32).clone(),
                "step": (f["step"].detach().cpu().clone() if torch.is_tensor(f["step"]) else torch.tensor(float(f["step"]))),
            }
    return {
        "format_version": FORMAT_VERSION,
        "completed_steps": int(completed_steps),
        "plan_version": int(plan_version),
        "identity": identity(config),
        "params": params,
        "optim": optim,
        "cpu_rng_state": cpu_rng,
        "cuda_rng_state": cuda_rng,
    }


def _torch_load(path: Path, mmap: bool = False) -> dict:
    return torch.load(path, weights_only=False, mmap=mmap)


def _same(a, b) -> bool:
    """Structural equality with tensors compared byte for byte (NaN payloads included)."""
    if torch.is_tensor(a):
        if not (torch.is_tensor(b) and a.dtype == b.dtype and a.shape == b.shape):
            return False
        return torch.equal(a.detach().contiguous().view(-1).view(torch.uint8),
                           b.detach().contiguous().view(-1).view(torch.uint8))
    if isinstance(a, dict):
        return isinstance(b, dict) and a.keys() == b.keys() and all(_same(a[k], b[k]) for k in a)
    if isinstance(a, (list, tuple)):
        return type(a) is type(b) and len(a) == len(b) and all(_same(x, y) for x, y in zip(a, b))
    return type(a) is type(b) and a == b


def _is_run(obj) -> bool:
    """A single-process run (:class:`resihp.reference.ReferenceRun`) rather than a config."""
    return hasattr(obj, "full_state") and hasattr(obj, "cursor") and hasattr(obj, "config")


def save_checkpoint(path, config: TrainConfig, full: dict | None = None, *, completed_steps: int | None = None,
                    plan_version: int = 0, rng: tuple | None = None) -> Path:
    """Atomically write the logical checkpoint; returns the canonical path.

    ``config`` + ``full`` (``{name: {param[, exp_avg, exp_avg_sq, step]}}``) +
    ``completed_steps``; or, as the reference calls it (``resihp/checkpoint.py:133``), a
    single-process run in place of ``config``, whose state and cursor are written.
    """
    if _is_run(config):
        run = config
        config, full = run.config, run.full_state()
        completed_steps = run.cursor if completed_steps is None else completed_steps
    if full is None or completed_steps is None:
        raise TypeError("save_checkpoint needs the full state and completed_steps (or a run)")
    if type(plan_version) is not int or plan_version < 0:
        raise CheckpointError("plan_version must be a non-negative integer")
    payload = build_payload(config, full, completed_steps=completed_steps, plan_version=plan_version, rng=rng)
    payload["digest"] = payload_digest(payload)
    path = Path(path)
    tmp = path.with_name(path.name + ".tmp")
    try:
        torch.save(payload, tmp)
        # read back and compare every field byte for byte with what was written (the
        # digest stored in it included): as strong as re-hashing, without a second SHA-256
        if not _same(_torch_load(tmp), payload):
            raise CheckpointError("checkpoint write verification failed: temp file differs from memory")
        os.replace(tmp, path)
    except BaseException:
        if tmp.exists():
            tmp.unlink()
        raise
    return path


class CheckpointWriter:
    """Writes checkpoints on a background thread, one at a time, in submission order.

    The gather that assembles the logical state stays a collective on the training
    ranks; only the writer rank's serialisation, read-back verification and atomic
    rename move off the iteration's critical path. :meth:`flush` waits for the write in
    flight and re-raises its error. Callers flush wherever the file must be current: at a
    safe point before any rank reads it, before a scheduled self-kill (so a fail-stop
    still happens after its iteration's commit, as in the reference), and at shutdown.
    """

    def __init__(self):
        self._thread = None
        self._error: BaseException | None = None
        self._pinned: dict[int, torch.Tensor] = {}
        self._stream = None

    def pinned(self, index: int, numel: int) -> torch.Tensor:
        """Page-locked FP32 staging buffer ``index`` of at least ``numel`` elements, reused
        across commits (callers flush before refilling it)."""
        buf = self._pinned.get(index)
        if buf is None or buf.numel() < numel:
            buf = torch.empty(numel, dtype=torch.float32, pin_memory=True)
            self._pinned[index] = buf
        return buf[:numel]

    def copy_stream(self, device):
        """The side stream the device-to-host copies of a commit run on."""
        if self._stream is None:
            self._stream = torch.cuda.Stream(device)
        return self._stream

    def submit(self, path, config: TrainConfig, full: dict, *, completed_steps: int, plan_version: int,
               ready=None) -> None:
        """Write ``full`` in the background; ``ready`` (a CUDA event) marks when its
        host tensors -- views of the pinned staging buffers -- hold their values."""
        import threading

        self.flush()
        rng = rng_states()  # as of the commit, not of the write

        def work():
            try:
                if ready is not None:
                    ready.synchronize()
                save_checkpoint(path, config, full, completed_steps=completed_steps, plan_version=plan_version,
                                rng=rng)
            except BaseException as error:  # re-raised by flush() on the training thread
                self._error = error

        self._thread = threading.Thread(target=work, name="resihp-checkpoint", daemon=True)
        self._thread.start()

    def flush(self) -> None:
        if self._thread is not None:
            self._thread.join()
            self._thread = None
        if self._error is not None:
            error, self._error = self._error, None
            raise error

    @property
    def pending(self) -> bool:
        return self._thread is not None and self._thread.is_alive()


def read_payload(path, *, mmap: bool = False) -> dict:
    path = Path(path)
    if not path.exists():
        raise CheckpointError(f"checkpoint missing: {path}")
    try:
        return _torch_load(path, mmap=mmap)
    except Exception as error:
        raise CheckpointError(f"checkpoint unreadable {path}: {error}") from error


def verify_digest(payload: dict) -> None:
    stored = payload.get("digest")
    if stored is None:
        raise CheckpointError("checkpoint has no content digest")
    if payload_digest(payload) != stored:
        raise CheckpointError("checkpoint digest mismatch: content is corrupted")


def validate(payload: dict, config: TrainConfig, expected_shapes: dict[str, tuple]) -> None:
    """Every structural check, each as its own root cause; the digest is checked last."""
    if payload.get("format_version") != FORMAT_VERSION:
        raise CheckpointError(f"unsupported checkpoint format version: {payload.get('format_version')}")
    if payload["identity"] != identity(config):
        raise CheckpointError(f"checkpoint identity differs from the run: {payload['identity']} != {identity(config)}")
    saved = payload["params"]
    missing = set(expected_shapes) - set(saved)
    if missing:
        raise CheckpointError(f"checkpoint is missing parameters: {sorted(missing)}")
    extra = set(saved) - set(expected_shapes)
    if extra:
        raise CheckpointError(f"checkpoint has unknown parameters: {sorted(extra)}")
    for name, shape in expected_shapes.items():
        if tuple(saved[name].shape) != tuple(shape):
            raise CheckpointError(f"checkpoint parameter shape mismatch {name}: {tuple(saved[name].shape)} != {tuple(shape)}")
    completed = payload["completed_steps"]
    optim = payload["optim"]
    if completed == 0:
        if optim:
            raise CheckpointError("cursor inconsistency: completed_steps is 0 but optimizer state is present")
    else:
        if set(optim) != set(saved):
            raise CheckpointError(
                f"cursor inconsistency: optimizer state does not match parameters "
                f"missing={sorted(set(saved) - set(optim))} extra={sorted(set(optim) - set(saved))}"
            )
        for name, state in optim.items():
            step = int(state["step"].item()) if torch.is_tensor(state["step"]) else int(state["step"])
            if step != completed:
                raise CheckpointError(f"cursor inconsistency: completed_steps={completed} but {name}.step={step}")
    verify_digest(payload)


def completed_steps(path) -> int:
    """The iterations a checkpoint has completed, read without loading its tensors."""
    return int(read_payload(path, mmap=True)["completed_steps"])


def load_anchor(path, *, verify: bool = True) -> tuple[dict[str, dict[str, torch.Tensor]], int]:
    """``({name: {param[, exp_avg, exp_avg_sq, step]}}, completed_steps)`` from a checkpoint."""
    payload = read_payload(path)
    if verify:
        verify_digest(payload)
    anchor = {}
    for name, param in payload["params"].items():
        entry = {"param": param}
        state = payload["optim"].get(name)
        if state is not None:
            entry.update({k: state[k] for k in OPTIM_STATES})
        anchor[name] = entry
    return anchor, payload["completed_steps"]


def install_anchor(model, optimizer, anchor: dict) -> None:
    """Load a full logical anchor into a module-form model and its ``torch.optim.AdamW``.

    ``model`` exposes ``logical_state_dict()`` (:class:`resihp.model.ReferenceTransformer`);
    ``anchor`` is :func:`load_anchor`'s ``{name: {param[, exp_avg, exp_avg_sq, step]}}``.
    Parameters and moments land on the model's device; the step count stays a CPU
    tensor, as torch's AdamW keeps it. Names the anchor has moments for replace the
    optimizer's whole state (reference: ``resihp/checkpoint.py:248-269``).
    """
    named = model.logical_state_dict()
    missing = sorted(set(named) - set(anchor))
    if missing:
        raise CheckpointError(f"anchor lacks parameters: {missing}")
    with torch.no_grad():
        for name, param in named.items():
            param.copy_(anchor[name]["param"].to(param.device, param.dtype))
    optimizer.state.clear()
    for name, param in named.items():
        fields = anchor[name]
        if "exp_avg" not in fields:
            continue
        step = fields["step"]
        optimizer.state[param] = {
            "step": (step.detach().clone() if torch.is_tensor(step) else torch.tensor(float(step))).to("cpu", torch.float32),
            "exp_avg": fields["exp_avg"].to(param.device, param.dtype).clone(),
            "exp_avg_sq": fields["exp_avg_sq"].to(param.device, param.dtype).clone(),
        }


def load_checkpoint(path, config: TrainConfig):
    """Validated ``(anchor, completed_steps, plan_version)``; restores the CPU/CUDA RNG.

    Given a single-process run instead of a config (the reference's call,
    ``resihp/checkpoint.py:272``), the state is installed into the run, its cursor set,
    and ``(completed_steps, plan_version)`` returned.
    """
    from .models.layout import model_specs

    run = config if _is_run(config) else None
    if run is not None:
        config = run.config
    payload = read_payload(path)
    validate(payload, config, {s.name: s.shape for s in model_specs(config)})
    torch.set_rng_state(payload["cpu_rng_state"])
    if payload["cuda_rng_state"] is not None and torch.cuda.is_available():
        torch.cuda.set_rng_state_all(payload["cuda_rng_state"])
    anchor, completed = load_anchor(path, verify=False)
    if run is not None:
        run.restore(anchor, completed)
        return completed, payload["plan_version"]
    return anchor, completed, payload["plan_version"]
