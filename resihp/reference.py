"""Single-process deterministic training run: the numerics oracle.

The token stream is the reference's exactly (``resihp/reference.py:97-103``): one
``torch.Generator`` seeded with ``config.seed`` draws ``randint(0, V, (B, S))`` per
iteration, so every rank of a distributed run and this oracle see the same batches. It
is generated lazily (a 1.3B-parameter run does not keep a thousand batches around).

:class:`ReferenceRun` trains the whole model as one stage at TP degree 1 on one device
with FP32 master weights -- the same :class:`~resihp.parallel.tp.TensorParallelStage`
code the distributed runtime uses -- on the full batch in one pass, and records the
loss plus SHA-256 digests of the parameters and AdamW state after every step.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass
from hashlib import sha256

import torch
from torch.nn import functional as F

from .config import TrainConfig, with_run_constants
from .models.init import initial_state
from .parallel.tp import TensorParallelStage

# AdamW and loss of a run whose config leaves them at their defaults (the reference's
# module constants, ``resihp/reference.py:20-23``); a config's own fields override them.
_DEFAULTS = {f.name: f.default for f in dataclasses.fields(TrainConfig)}
LEARNING_RATE = _DEFAULTS["lr"]
WEIGHT_DECAY = _DEFAULTS["weight_decay"]
ADAM_BETAS = (_DEFAULTS["beta1"], _DEFAULTS["beta2"])
ADAM_EPS = _DEFAULTS["adam_eps"]


def adamw(params, config: TrainConfig | None = None) -> torch.optim.AdamW:
    """``torch.optim.AdamW`` over ``params`` with ``config``'s hyper-parameters (default:
    the module constants) -- the optimizer a module-form model trains with to match a run.
    """
    if config is None:
        return torch.optim.AdamW(params, lr=LEARNING_RATE, betas=ADAM_BETAS, eps=ADAM_EPS, weight_decay=WEIGHT_DECAY)
    return torch.optim.AdamW(params, lr=config.lr, betas=(config.beta1, config.beta2), eps=config.adam_eps,
                             weight_decay=config.weight_decay)


def next_token_loss(logits: torch.Tensor, tokens: torch.Tensor, vocab_size: int) -> torch.Tensor:
    """Mean cross-entropy of ``logits [B, S, V]`` against the next token of ``tokens [B, S]``."""
    return F.cross_entropy(logits[:, :-1].reshape(-1, vocab_size), tokens[:, 1:].reshape(-1))


class TokenStream:
    """Batch ``i`` of the fixed, seeded data order (``randint(0, V, (B, S))`` per step)."""

    def __init__(self, vocab_size: int, sequence_length: int, batch_size: int, seed: int, *, pin: bool = False):
        self.shape = (batch_size, sequence_length)
        self.vocab_size = vocab_size
        self.seed = seed
        self.pin = pin
        self._gen = torch.Generator().manual_seed(seed)
        self._next = 0
        self._cache: dict[int, torch.Tensor] = {}

    def __getitem__(self, index: int) -> torch.Tensor:
        if index in self._cache:
            return self._cache[index]
        if index < self._next:
            self._gen = torch.Generator().manual_seed(self.seed)
            self._next = 0
        batch = None
        while self._next <= index:
            batch = torch.randint(0, self.vocab_size, self.shape, generator=self._gen)
            self._next += 1
        if self.pin and torch.cuda.is_available():
            batch = batch.pin_memory()
        self._cache = {index: batch}
        return batch


def token_stream(config: TrainConfig, *, pin: bool = False) -> TokenStream:
    return TokenStream(config.vocab_size, config.seq_len, config.batch_size, config.seed, pin=pin)


def digest_tensors(items) -> str:
    """SHA-256 over ``(name, tensor)`` pairs by their exact FP32 bytes."""
    h = sha256()
    for name, tensor in items:
        arr = tensor.detach().cpu().to(torch.float32).contiguous().numpy()
        h.update(name.encode("utf-8"))
        h.update(repr(arr.shape).encode("utf-8"))
        h.update(arr.tobytes())
    return h.hexdigest()


def logical_state_digest(model) -> str:
    """SHA-256 of a model's full logical parameters, for anything with
    ``logical_state_dict()`` (a stage at TP degree 1, a module-form model)."""
    return digest_tensors(sorted(model.logical_state_dict().items()))


@dataclass(frozen=True)
class StepRecord:
    step: int
    loss: float
    param_digest: str
    optim_digest: str
    tokens: tuple = ()  # the batch, row by row (the reference records it too)


class ReferenceRun:
    """The whole model in one process (see the module docstring)."""

    def __init__(self, config: TrainConfig, *, device="cpu", full_state=None, moments=None, cursor: int = 0,
                 vocab_size: int | None = None, sequence_length: int | None = None):
        config = with_run_constants(config, vocab_size, sequence_length)  # the reference's run constants
        if config.seq_len < 2:
            raise ValueError("sequence_length must be at least 2 for next-token loss")
        self.config = config
        self.vocab_size = config.vocab_size
        self.sequence_length = config.seq_len
        self.device = torch.device(device)
        state = initial_state(config, device=self.device) if full_state is None else full_state
        self.stage = TensorParallelStage(
            config, layer_ids=range(config.num_layers), is_first=True, is_last=True,
            local_state=state, group=None, device=self.device, moments=moments,
        )
        self.batches = token_stream(config)
        self.cursor = cursor

    def step(self) -> StepRecord:
        tokens = self.batches[self.cursor].to(self.device)
        stage = self.stage
        stage.zero_grad()
        b, s = tokens.shape
        loss = stage.forward(tokens=tokens, loss_scale=1.0 / (b * (s - 1)))
        loss.backward()
        stage.optimizer_step()
        record = StepRecord(
            step=self.cursor,
            tokens=tuple(tuple(row) for row in tokens.tolist()),
            loss=float(loss.detach()),
            param_digest=digest_tensors(sorted(stage.logical_state_dict().items())),
            optim_digest=digest_tensors(sorted(
                (f"{n}.{k}", v) for n in stage.logical_state_dict() for k, v in stage.moment_views(n).items()
            )),
        )
        self.cursor += 1
        return record

    def restore(self, anchor: dict, completed: int) -> None:
        """Install a full logical anchor (``{name: {param[, exp_avg, exp_avg_sq, step]}}``)
        and continue after ``completed`` steps."""
        stage = self.stage
        with torch.no_grad():
            for name, view in stage.logical_state_dict().items():
                view.copy_(anchor[name]["param"].to(view.device, torch.float32))
            stage.flat.exp_avg.zero_()
            stage.flat.exp_avg_sq.zero_()
            stage.flat.step = 0
        stage.install_moments({n: e for n, e in anchor.items() if "exp_avg" in e})
        stage.flat.refresh_work()
        self.cursor = int(completed)

    def full_state(self) -> dict[str, dict[str, torch.Tensor]]:
        """``{name: {param, exp_avg, exp_avg_sq, step}}`` (the checkpoint's logical form)."""
        out = {}
        step = torch.tensor(float(self.stage.flat.step))
        for name, (view, _d) in self.stage.local_shards().items():
            entry = {"param": view.detach().clone()}
            if self.stage.flat.step > 0:
                mv = self.stage.moment_views(name)
                entry.update({k: v.detach().clone() for k, v in mv.items()})
                entry["step"] = step.clone()
            out[name] = entry
        return out


def run_reference(config: TrainConfig, *, device="cpu", vocab_size: int | None = None,
                  sequence_length: int | None = None) -> list[StepRecord]:
    run = ReferenceRun(config, device=device, vocab_size=vocab_size, sequence_length=sequence_length)
    return [run.step() for _ in range(run.config.iterations)]
