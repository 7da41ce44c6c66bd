"""Logical tensors of the two decoder architectures: names, shapes, TP shard dims.

A logical tensor keeps one stable name for the whole run (``layers.<gid>.<suffix>``
with the global layer id), whatever stage owns it and at whatever TP degree -- the
identity the checkpoint, the state routes and the reshard all speak. This module is
the single source of truth for the shard layout (reference: ``resihp/parallel/
reshard.py:41-81``): dim 0 = column-parallel (output features / vocabulary / heads),
dim 1 = row-parallel (input features), ``None`` = replicated.

GPT-2 blocks (``arch="gpt2"``) use the reference's names; Llama blocks use
``attn.{q,k,v,o}_proj``, ``mlp.{gate,up,down}`` and RMSNorm weights. With tied
embeddings there is no ``lm_head.weight``: the last stage's head group carries a copy
of ``token_embedding.weight`` instead.
"""

from __future__ import annotations

from dataclasses import dataclass

from ..config import TrainConfig


@dataclass(frozen=True)
class TensorSpec:
    name: str
    shape: tuple[int, ...]          # full logical shape
    shard_dim: int | None           # TP shard dim, None = replicated
    init: str                       # "normal" | "ones" | "zeros"
    fuse: str = ""                  # local fused-buffer group ("qkv", "gate_up") or ""


def layer_specs(config: TrainConfig, gid: int) -> list[TensorSpec]:
    d = config.model_dim
    p = f"layers.{gid}."
    if config.arch == "gpt2":
        return [
            TensorSpec(p + "attn_norm.weight", (d,), None, "ones"),
            TensorSpec(p + "attn_norm.bias", (d,), None, "zeros"),
            TensorSpec(p + "attn.q_proj.weight", (d, d), 0, "normal"),
            TensorSpec(p + "attn.k_proj.weight", (d, d), 0, "normal"),
            TensorSpec(p + "attn.v_proj.weight", (d, d), 0, "normal"),
            TensorSpec(p + "attn.out_proj.weight", (d, d), 1, "normal"),
            TensorSpec(p + "mlp_norm.weight", (d,), None, "ones"),
            TensorSpec(p + "mlp_norm.bias", (d,), None, "zeros"),
            TensorSpec(p + "mlp.fc1.weight", (config.ffn, d), 0, "normal"),
            TensorSpec(p + "mlp.fc2.weight", (d, config.ffn), 1, "normal"),
        ]
    hd = config.head_dim
    q = config.num_heads * hd
    kv = config.kv_heads * hd
    f = config.ffn
    return [
        TensorSpec(p + "attn_norm.weight", (d,), None, "ones"),
        TensorSpec(p + "attn.q_proj.weight", (q, d), 0, "normal", "qkv"),
        TensorSpec(p + "attn.k_proj.weight", (kv, d), 0, "normal", "qkv"),
        TensorSpec(p + "attn.v_proj.weight", (kv, d), 0, "normal", "qkv"),
        TensorSpec(p + "attn.o_proj.weight", (d, q), 1, "normal"),
        TensorSpec(p + "mlp_norm.weight", (d,), None, "ones"),
        TensorSpec(p + "mlp.gate.weight", (f, d), 0, "normal", "gate_up"),
        TensorSpec(p + "mlp.up.weight", (f, d), 0, "normal", "gate_up"),
        TensorSpec(p + "mlp.down.weight", (d, f), 1, "normal"),
    ]


def embedding_specs(config: TrainConfig) -> list[TensorSpec]:
    out = [TensorSpec("token_embedding.weight", (config.vocab_size, config.model_dim), 0, "normal")]
    if config.arch == "gpt2":
        out.append(TensorSpec("position_embedding.weight", (config.seq_len, config.model_dim), None, "normal"))
    return out


def head_specs(config: TrainConfig) -> list[TensorSpec]:
    d = config.model_dim
    out = [TensorSpec("final_norm.weight", (d,), None, "ones")]
    if config.arch == "gpt2":
        out.append(TensorSpec("final_norm.bias", (d,), None, "zeros"))
    if config.tied_embeddings:
        out.append(TensorSpec("token_embedding.weight", (config.vocab_size, d), 0, "normal"))
    else:
        out.append(TensorSpec("lm_head.weight", (config.vocab_size, d), 0, "normal"))
    return out


def group_specs(config: TrainConfig, layer: int | None, boundary: str) -> list[TensorSpec]:
    """Specs of one routable state group (a layer, or the embedding/head boundary)."""
    if boundary == "embedding":
        return embedding_specs(config)
    if boundary == "head":
        return head_specs(config)
    return layer_specs(config, layer)


def stage_specs(config: TrainConfig, layer_ids, is_first: bool, is_last: bool) -> list[TensorSpec]:
    """Everything one stage holds, in canonical order, each name once."""
    out: list[TensorSpec] = []
    seen: set[str] = set()

    def add(specs):
        for s in specs:
            if s.name not in seen:
                seen.add(s.name)
                out.append(s)

    if is_first:
        add(embedding_specs(config))
    for gid in layer_ids:
        add(layer_specs(config, gid))
    if is_last:
        add(head_specs(config))
    return out


def model_specs(config: TrainConfig) -> list[TensorSpec]:
    return stage_specs(config, range(config.num_layers), True, True)


def shard_dims(config: TrainConfig, layer_ids=None) -> dict[str, int | None]:
    """Logical name -> shard dim for the whole model (or the given layers + boundaries)."""
    ids = range(config.num_layers) if layer_ids is None else layer_ids
    return {s.name: s.shard_dim for s in stage_specs(config, ids, True, True)}


def local_shape(spec: TensorSpec, tp_size: int) -> tuple[int, ...]:
    if spec.shard_dim is None or tp_size == 1:
        return spec.shape
    shape = list(spec.shape)
    if shape[spec.shard_dim] % tp_size:
        raise ValueError(f"{spec.name}: dim {spec.shard_dim} of {spec.shape} does not split {tp_size} ways")
    shape[spec.shard_dim] //= tp_size
    return tuple(shape)


def parameter_count(config: TrainConfig) -> int:
    total = 0
    for s in model_specs(config):
        n = 1
        for x in s.shape:
            n *= x
        total += n
    return total


def kernel_shape_problems(config: TrainConfig, tp_size: int) -> list[str]:
    """The shape rules of the bf16 sm_100a kernels that a stage at TP degree ``tp_size``
    would break (empty when the shape runs). The same rules the kernels' host wrappers
    check before a launch (``csrc/attention.cu``, ``norm.cu``, ``xent.cu``, ``gemm.cu``),
    gathered so a stage can refuse an unsupported shape with one message at set-up."""
    out = []
    d, hd, tp = config.model_dim, config.head_dim, tp_size
    if hd not in (64, 128):
        out.append(f"head_dim {hd} (attention: 64 or 128)")
    if config.seq_len % 128:
        out.append(f"seq_len {config.seq_len} (attention: a multiple of 128)")
    w = d // 8
    if d % 8 or w == 0 or w > 1024 or (w % 32 if w >= 32 else 32 % w):
        out.append(f"model_dim {d} (RMSNorm: a multiple of 8, at most 8192, d/8 dividing or divisible by 32)")
    if (config.vocab_size // tp) % 8:
        out.append(f"vocabulary shard {config.vocab_size // tp} (cross-entropy and LM-head GEMM: a multiple of 8)")
    hq, hkv = config.num_heads // tp, config.kv_heads // tp
    for what, n in (("fused QKV width", (hq + 2 * hkv) * hd), ("attention output width", hq * hd),
                    ("FFN shard", config.ffn // tp)):
        if n % 8:
            out.append(f"{what} {n} (GEMM operands: a multiple of 8)")
    return out
