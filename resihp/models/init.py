"""Deterministic initial weights for a configuration.

* GPT-2 blocks: the reference's module construction order and torch defaults
  (``resihp/model.py:100-116``: embeddings ``normal(0, 1)``, ``nn.Linear``
  Kaiming-uniform, LayerNorm ones/zeros), driven by ``torch.manual_seed(seed)``, so the
  full logical state is bit-identical to the reference model built with the same seed.
* Llama blocks: every matrix ``normal(0, init_std)`` (default 0.02), norm weights 1.
  Each logical tensor is drawn from CPU generators seeded from ``(seed, name)`` (a large
  tensor in fixed 4 Mi-element pieces, each with its own seed, drawn on a thread pool)
  and then moved to the device it trains on. A rank therefore materialises only the
  tensors its stage owns and still agrees bit for bit with every other rank, with a
  single-process run, and with a run on another device type: the CUDA and CPU
  generators produce different streams from one seed, so a draw on the training
  device would make the initial model depend on where it is trained.
"""

from __future__ import annotations

import zlib
from concurrent.futures import ThreadPoolExecutor

import torch

from ..config import TrainConfig
from .layout import TensorSpec, model_specs, stage_specs


def _gpt2_reference_state(config: TrainConfig) -> dict[str, torch.Tensor]:
    d = config.model_dim
    # The reference seeds the global generator (``torch.manual_seed``) before building its
    # modules; only the CPU stream feeds these draws, so only the CPU generator is
    # reseeded, and its state is put back afterwards: a draw in the middle of a run (a
    # rollback to the initial state) leaves the run's own random streams untouched.
    saved = torch.get_rng_state()
    torch.random.default_generator.manual_seed(config.seed)
    try:
        return _gpt2_modules_state(config, d)
    finally:
        torch.set_rng_state(saved)


def _gpt2_modules_state(config: TrainConfig, d: int) -> dict[str, torch.Tensor]:
    from torch import nn

    state: dict[str, torch.Tensor] = {}
    state["token_embedding.weight"] = nn.Embedding(config.vocab_size, d).weight.detach()
    state["position_embedding.weight"] = nn.Embedding(config.seq_len, d).weight.detach()
    for gid in range(config.num_layers):
        p = f"layers.{gid}."
        state[p + "attn_norm.weight"] = nn.LayerNorm(d).weight.detach()
        state[p + "attn_norm.bias"] = torch.zeros(d)
        for name in ("q_proj", "k_proj", "v_proj", "out_proj"):
            state[p + f"attn.{name}.weight"] = nn.Linear(d, d, bias=False).weight.detach()
        state[p + "mlp_norm.weight"] = nn.LayerNorm(d).weight.detach()
        state[p + "mlp_norm.bias"] = torch.zeros(d)
        state[p + "mlp.fc1.weight"] = nn.Linear(d, config.ffn, bias=False).weight.detach()
        state[p + "mlp.fc2.weight"] = nn.Linear(config.ffn, d, bias=False).weight.detach()
    state["final_norm.weight"] = nn.LayerNorm(d).weight.detach()
    state["final_norm.bias"] = torch.zeros(d)
    head = nn.Linear(d, config.vocab_size, bias=False).weight.detach()
    if config.tied_embeddings:
        pass  # the head reuses token_embedding.weight
    else:
        state["lm_head.weight"] = head
    return state


def _seed_for(config: TrainConfig, name: str) -> int:
    return (config.seed * 1_000_003 + zlib.crc32(name.encode("utf-8"))) & 0x7FFF_FFFF_FFFF


# Elements drawn per CPU generator. A tensor up to this size is one generator's stream
# (its values do not depend on the piece size); a larger one is cut into pieces of this
# many elements in row-major order, piece i seeded from ``(seed, name#i)``.
DRAW_PIECE = 1 << 22


def _draw_normal(config: TrainConfig, name: str, numel: int) -> torch.Tensor:
    out = torch.empty(numel, dtype=torch.float32)
    if numel <= DRAW_PIECE:
        gen = torch.Generator().manual_seed(_seed_for(config, name))
        return torch.randn(numel, generator=gen, out=out)

    def piece(i: int) -> None:
        lo = i * DRAW_PIECE
        chunk = out[lo:lo + DRAW_PIECE]
        gen = torch.Generator().manual_seed(_seed_for(config, f"{name}#{i}"))
        torch.randn(chunk.numel(), generator=gen, out=chunk)

    n_pieces = (numel + DRAW_PIECE - 1) // DRAW_PIECE
    with ThreadPoolExecutor(max_workers=min(16, n_pieces)) as pool:
        list(pool.map(piece, range(n_pieces)))
    return out


def init_tensor(config: TrainConfig, spec: TensorSpec, device) -> torch.Tensor:
    """One Llama-block logical tensor, full shape, FP32, on ``device``; its values do
    not depend on ``device`` (drawn on the CPU, then moved)."""
    if spec.init == "ones":
        return torch.ones(spec.shape, dtype=torch.float32, device=device)
    if spec.init == "zeros":
        return torch.zeros(spec.shape, dtype=torch.float32, device=device)
    numel = 1
    for n in spec.shape:
        numel *= n
    std = 0.02 if config.init_std is None else config.init_std
    values = _draw_normal(config, spec.name, numel).view(spec.shape).mul_(std)
    return values.to(device)


def initial_state(config: TrainConfig, *, names=None, device="cpu") -> dict[str, torch.Tensor]:
    """Full logical FP32 tensors for ``names`` (default: the whole model)."""
    if config.arch == "gpt2":
        full = _gpt2_reference_state(config)
        keep = full if names is None else {n: full[n] for n in names}
        return {n: t.to(device) for n, t in keep.items()}
    specs = {s.name: s for s in model_specs(config)}
    wanted = list(specs) if names is None else list(names)
    return {n: init_tensor(config, specs[n], device) for n in wanted}


def initial_stage_state(config: TrainConfig, layer_ids, is_first, is_last, device="cpu") -> dict[str, torch.Tensor]:
    names = [s.name for s in stage_specs(config, layer_ids, is_first, is_last)]
    return initial_state(config, names=names, device=device)
