"""The one analytical memory model every planning decision gates on.

Two regimes share one entry point:

* **Reference regime** (``arch="gpt2"``, ``dtype="fp32"``): byte-for-byte the
  reference formula (``resihp/memory.py:40-102``): per layer ``12d^2+4d`` FP32
  parameters sharded over TP, a ``2Vd`` embedding/head term sharded over TP, gradient
  and both Adam moments equal to the parameter bytes, and a deliberately lower-bound
  activation term of ``tokens * d * 4 * (1/TP + 1)`` for one layer. Keeping it exact is
  what lets this planner reproduce the reference's plans (and plan digests) wherever
  the reference can express the configuration.
* **B200 regime** (everything else, i.e. Llama blocks and/or bf16): weights in the
  compute dtype plus an FP32 master copy when that dtype is bf16, FP32 gradient
  accumulation buffers (two on the bf16 GPU path) and FP32 Adam moments, the fused TP
  workspace under sequence parallelism, and a *per-layer* activation model that
  follows what the runtime actually keeps alive between a micro-batch's forward and its
  backward: the normalised inputs, Q/K/V after RoPE, the attention output and its
  log-sum-exp, both MLP projections and the SwiGLU product. Under sequence parallelism
  the block input and residual shrink by TP while the two column-parallel GEMM inputs
  are kept gathered; with recompute only each block's input
  is kept, plus one block's full working set while it is being recomputed. The last
  stage adds one micro-batch of FP32 vocab-parallel logits.

``in_flight_micro_batches`` has no default on purpose: callers replay the 1F1B schedule
(:func:`resihp.planner.pp.peak_in_flight`) so that the model and the runtime agree on
the activation peak.
"""

from __future__ import annotations

from dataclasses import dataclass

from .config import TrainConfig
from .validate import positive_int

FP32 = 4
BF16 = 2


@dataclass(frozen=True)
class MemoryBreakdown:
    sharded_parameters: int
    boundary_parameters: int
    gradients: int
    adam_exp_avg: int
    adam_exp_avg_sq: int
    activation: int

    @property
    def total(self) -> int:
        return (
            self.sharded_parameters + self.boundary_parameters + self.gradients
            + self.adam_exp_avg + self.adam_exp_avg_sq + self.activation
        )


def layer_parameter_count(config: TrainConfig) -> tuple[int, int]:
    """``(tp-sharded, replicated)`` parameter counts of one transformer block."""
    d = config.model_dim
    if config.arch == "gpt2":
        # q,k,v,o + fc1/fc2 matrices; two LayerNorms with weight and bias.
        return 4 * d * d + 2 * d * config.ffn, 4 * d
    kv = config.kv_heads * config.head_dim
    return d * d + 2 * d * kv + d * d + 3 * d * config.ffn, 2 * d


def _reference_regime(config: TrainConfig) -> bool:
    return config.arch == "gpt2" and config.dtype == "fp32"


def estimate_memory(
    config: TrainConfig,
    *,
    tp_degree: int,
    stage_layers: int,
    micro_batches: int,
    sequence_length: int,
    vocab_size: int,
    in_flight_micro_batches: int,
) -> MemoryBreakdown:
    """Resident bytes of one pipeline stage on one TP rank."""
    for name, value in (
        ("tp_degree", tp_degree), ("stage_layers", stage_layers),
        ("micro_batches", micro_batches), ("sequence_length", sequence_length),
        ("vocab_size", vocab_size), ("in_flight_micro_batches", in_flight_micro_batches),
    ):
        positive_int(name, value)
    if in_flight_micro_batches > micro_batches:
        raise ValueError("in_flight_micro_batches cannot exceed micro_batches")
    d = config.model_dim
    if d % tp_degree or config.num_heads % tp_degree:
        raise ValueError("tp_degree must divide model_dim and num_heads")
    tokens = in_flight_micro_batches * config.micro_batch_size * sequence_length

    if _reference_regime(config):
        sharded_count, replicated_count = layer_parameter_count(config)
        per_layer = sharded_count + replicated_count
        sharded = stage_layers * per_layer * FP32 // tp_degree
        boundary = 2 * vocab_size * d * FP32 // tp_degree
        grads = sharded + boundary
        activation = tokens * d * FP32 // tp_degree + tokens * d * FP32
        return MemoryBreakdown(sharded, boundary, grads, grads, grads, activation)

    act = BF16 if config.dtype == "bf16" else FP32
    weight_bytes = act + (FP32 if config.dtype == "bf16" else 0)  # + fp32 master
    sharded_count, replicated_count = layer_parameter_count(config)
    layer_params = sharded_count // tp_degree + replicated_count
    stage_params = stage_layers * layer_params
    boundary_params = 2 * vocab_size * d // tp_degree
    sharded = stage_params * weight_bytes
    boundary = boundary_params * weight_bytes
    # bf16 runs on the GPU path, which keeps two FP32 gradient buffers (the fused DP step
    # reads one and writes the reduced sum into the other)
    grad_buffers = 2 if config.dtype == "bf16" else 1
    grads = (stage_params + boundary_params) * FP32 * grad_buffers
    moments = (stage_params + boundary_params) * FP32

    kv = config.kv_heads * config.head_dim
    sp = tp_degree if config.sequence_parallel else 1
    # block input and residual stay token-sharded under SP; the inputs of the two
    # column-parallel GEMMs (attention norm and MLP norm outputs) are kept gathered over
    # the full sequence for their weight gradients
    replicated_terms = 2 * d * act // sp + 2 * d * act
    sharded_terms = ((d + 2 * kv) + d + 3 * config.ffn) * act // tp_degree
    lse = (config.num_heads // tp_degree) * FP32
    full_block = replicated_terms + sharded_terms + lse
    mb_tokens = config.micro_batch_size * sequence_length
    if config.recompute:
        per_token = d * act // sp
        activation = tokens * stage_layers * per_token + mb_tokens * full_block
    else:
        activation = tokens * stage_layers * full_block
    activation += mb_tokens * (vocab_size // tp_degree) * FP32
    if config.dtype == "bf16" and config.sequence_parallel and tp_degree > 1:
        # the fused TP kernels' peer-memory workspace: two publish slots, two partial
        # buffers and one receive buffer of one micro-batch
        activation += (2 * mb_tokens // tp_degree + 3 * mb_tokens) * d * BF16
    return MemoryBreakdown(sharded, boundary, grads, moments, moments, activation)


def memory_feasible(
    config: TrainConfig,
    *,
    tp_degree: int,
    stage_layers: int,
    micro_batches: int,
    sequence_length: int,
    vocab_size: int,
    memory_budget: int,
    in_flight_micro_batches: int,
) -> bool:
    positive_int("memory_budget", memory_budget)
    return estimate_memory(
        config,
        tp_degree=tp_degree,
        stage_layers=stage_layers,
        micro_batches=micro_batches,
        sequence_length=sequence_length,
        vocab_size=vocab_size,
        in_flight_micro_batches=in_flight_micro_batches,
    ).total <= memory_budget
