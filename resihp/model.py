"""The decoder as a ``torch.nn`` module tree whose parameter names are the logical names.

The training runtime keeps a stage's parameters in one flat FP32 state and runs the
decoder as a chain of fused ops (:class:`resihp.parallel.tp.TensorParallelStage`).
This module builds the same two architectures from ordinary modules -- ``nn.Linear``,
``nn.LayerNorm`` / ``nn.RMSNorm``, ``nn.Embedding`` and torch's scaled-dot-product
attention -- for code that wants a model object (inspection, export, a plain
``torch.optim`` loop), and as an FP32 oracle that shares none of the runtime's ops:
its loss and gradients must match the stage's.

Reference API (``resihp/model.py:44-137``): ``MLP_RATIO``, ``CausalSelfAttention``,
``MLP``, ``TransformerBlock`` and ``ReferenceTransformer`` with ``layer_ids``,
``forward(tokens) -> logits`` and ``logical_state_dict()``. The layers sit in an
``nn.ModuleDict`` keyed by the global layer id, so ``named_parameters()`` yields
exactly the names of :func:`resihp.models.layout.model_specs` (``layers.<gid>.<...>``)
and a checkpoint anchor or an initial state loads by name. A new model starts from
:func:`resihp.models.init.initial_state`, the init every run of the same config uses.

Llama blocks add ``GroupedQueryAttention`` (GQA, rotate-half RoPE), ``SwiGLU`` and
``LlamaBlock``; with ``tied_embeddings`` the head multiplies by the token embedding and
there is no ``lm_head.weight``.
"""

from __future__ import annotations

import torch
from torch import nn
from torch.nn import functional as F

from .config import TrainConfig, with_run_constants
from .models.init import initial_state

#: GPT-2 blocks: MLP hidden width as a multiple of ``model_dim`` (``ffn_dim`` overrides).
MLP_RATIO = 4


def _split_heads(y, heads: int):
    """``[B, S, heads * D]`` -> ``[B, heads, S, D]``."""
    b, s, _ = y.shape
    return y.view(b, s, heads, -1).transpose(1, 2)


class CausalSelfAttention(nn.Module):
    """GPT-2 multi-head causal self-attention (bias-free ``q/k/v/out_proj``)."""

    def __init__(self, model_dim: int, num_heads: int):
        super().__init__()
        if model_dim % num_heads:
            raise ValueError("model_dim must be divisible by num_heads")
        self.num_heads = num_heads
        self.head_dim = model_dim // num_heads
        self.q_proj = nn.Linear(model_dim, model_dim, bias=False)
        self.k_proj = nn.Linear(model_dim, model_dim, bias=False)
        self.v_proj = nn.Linear(model_dim, model_dim, bias=False)
        self.out_proj = nn.Linear(model_dim, model_dim, bias=False)

    def forward(self, x):
        b, s, _ = x.shape
        q = _split_heads(self.q_proj(x), self.num_heads)
        k = _split_heads(self.k_proj(x), self.num_heads)
        v = _split_heads(self.v_proj(x), self.num_heads)
        ctx = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.out_proj(ctx.transpose(1, 2).reshape(b, s, -1))


class RotaryEmbedding(nn.Module):
    """Rotate-half RoPE: channel pair ``(i, i + D/2)`` turns by ``pos * theta^(-2i/D)``."""

    def __init__(self, head_dim: int, max_positions: int, theta: float):
        super().__init__()
        if head_dim % 2:
            raise ValueError("RoPE needs an even head_dim")
        exponent = torch.arange(head_dim // 2, dtype=torch.float64) * (2.0 / head_dim)
        angle = torch.arange(max_positions, dtype=torch.float64)[:, None] * torch.pow(theta, -exponent)[None, :]
        self.register_buffer("cos", angle.cos().float(), persistent=False)
        self.register_buffer("sin", angle.sin().float(), persistent=False)

    def forward(self, x):  # x: [B, H, S, D]
        s = x.shape[2]
        cos, sin = self.cos[:s], self.sin[:s]
        a, b = x.chunk(2, dim=-1)
        return torch.cat([a * cos - b * sin, b * cos + a * sin], dim=-1)


class GroupedQueryAttention(nn.Module):
    """Llama causal attention: ``num_kv_heads`` K/V heads shared by groups of Q heads,
    RoPE on Q and K, output projection ``o_proj``."""

    def __init__(self, model_dim: int, num_heads: int, num_kv_heads: int, *, max_positions: int, theta: float):
        super().__init__()
        if model_dim % num_heads or num_heads % num_kv_heads:
            raise ValueError("model_dim must divide by num_heads and num_heads by num_kv_heads")
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = model_dim // num_heads
        kv = num_kv_heads * self.head_dim
        self.q_proj = nn.Linear(model_dim, model_dim, bias=False)
        self.k_proj = nn.Linear(model_dim, kv, bias=False)
        self.v_proj = nn.Linear(model_dim, kv, bias=False)
        self.o_proj = nn.Linear(model_dim, model_dim, bias=False)
        self.rope = RotaryEmbedding(self.head_dim, max_positions, theta)

    def forward(self, x):
        b, s, _ = x.shape
        q = self.rope(_split_heads(self.q_proj(x), self.num_heads))
        k = self.rope(_split_heads(self.k_proj(x), self.num_kv_heads))
        v = _split_heads(self.v_proj(x), self.num_kv_heads)
        ctx = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=self.num_kv_heads != self.num_heads)
        return self.o_proj(ctx.transpose(1, 2).reshape(b, s, -1))


class MLP(nn.Module):
    """GPT-2 MLP: ``fc2(gelu(fc1 x))``, bias-free."""

    def __init__(self, model_dim: int, hidden: int | None = None):
        super().__init__()
        hidden = MLP_RATIO * model_dim if hidden is None else hidden
        self.fc1 = nn.Linear(model_dim, hidden, bias=False)
        self.fc2 = nn.Linear(hidden, model_dim, bias=False)

    def forward(self, x):
        return self.fc2(F.gelu(self.fc1(x)))


class SwiGLU(nn.Module):
    """Llama MLP: ``down(silu(gate x) * up x)``, bias-free."""

    def __init__(self, model_dim: int, hidden: int):
        super().__init__()
        self.gate = nn.Linear(model_dim, hidden, bias=False)
        self.up = nn.Linear(model_dim, hidden, bias=False)
        self.down = nn.Linear(hidden, model_dim, bias=False)

    def forward(self, x):
        return self.down(F.silu(self.gate(x)) * self.up(x))


class TransformerBlock(nn.Module):
    """GPT-2 pre-norm block: ``x + attn(ln(x))``, then ``x + mlp(ln(x))``."""

    def __init__(self, model_dim: int, num_heads: int, *, ffn_dim: int | None = None):
        super().__init__()
        self.attn_norm = nn.LayerNorm(model_dim)
        self.attn = CausalSelfAttention(model_dim, num_heads)
        self.mlp_norm = nn.LayerNorm(model_dim)
        self.mlp = MLP(model_dim, ffn_dim)

    def forward(self, x):
        x = x + self.attn(self.attn_norm(x))
        return x + self.mlp(self.mlp_norm(x))


class LlamaBlock(nn.Module):
    """Llama pre-norm block: RMSNorm, GQA + RoPE, RMSNorm, SwiGLU."""

    def __init__(self, config: TrainConfig):
        super().__init__()
        d = config.model_dim
        self.attn_norm = nn.RMSNorm(d, eps=config.norm_eps)
        self.attn = GroupedQueryAttention(d, config.num_heads, config.kv_heads, max_positions=config.seq_len,
                                          theta=config.rope_theta)
        self.mlp_norm = nn.RMSNorm(d, eps=config.norm_eps)
        self.mlp = SwiGLU(d, config.ffn)

    def forward(self, x):
        x = x + self.attn(self.attn_norm(x))
        return x + self.mlp(self.mlp_norm(x))


class ReferenceTransformer(nn.Module):
    """The whole decoder for ``config`` (GPT-2 or Llama blocks), FP32.

    ``vocab_size`` / ``sequence_length`` default to the config's; passing them (the
    reference's signature) overrides the config's token-stream shape. ``init=False``
    leaves torch's module defaults instead of loading the run's initial state.
    """

    def __init__(self, config: TrainConfig, *, vocab_size: int | None = None, sequence_length: int | None = None,
                 init: bool = True):
        super().__init__()
        config = with_run_constants(config, vocab_size, sequence_length)
        self.config = config
        self.vocab_size = config.vocab_size
        self.sequence_length = config.seq_len
        d = config.model_dim
        self.token_embedding = nn.Embedding(config.vocab_size, d)
        gpt2 = config.arch == "gpt2"
        if gpt2:
            self.position_embedding = nn.Embedding(config.seq_len, d)
        self.layers = nn.ModuleDict({
            str(gid): (TransformerBlock(d, config.num_heads, ffn_dim=config.ffn) if gpt2 else LlamaBlock(config))
            for gid in range(config.num_layers)
        })
        self.final_norm = nn.LayerNorm(d) if gpt2 else nn.RMSNorm(d, eps=config.norm_eps)
        if not config.tied_embeddings:
            self.lm_head = nn.Linear(d, config.vocab_size, bias=False)
        if init:
            self.load_logical_state(initial_state(config))

    @property
    def layer_ids(self) -> tuple[int, ...]:
        """Global layer ids in execution order (the ``ModuleDict`` keys, not a range)."""
        return tuple(sorted(int(gid) for gid in self.layers))

    def forward(self, tokens):
        """``tokens [B, S]`` -> logits ``[B, S, V]``."""
        _, s = tokens.shape
        if s != self.sequence_length:
            raise ValueError("token sequence length does not match the model")
        x = self.token_embedding(tokens)
        if self.config.arch == "gpt2":
            x = x + self.position_embedding(torch.arange(s, device=tokens.device))
        for gid in self.layer_ids:
            x = self.layers[str(gid)](x)
        x = self.final_norm(x)
        if self.config.tied_embeddings:
            return F.linear(x, self.token_embedding.weight)
        return self.lm_head(x)

    def loss(self, tokens):
        """Mean next-token cross-entropy of ``tokens`` (the training objective)."""
        logits = self(tokens)
        return F.cross_entropy(logits[:, :-1].reshape(-1, self.vocab_size), tokens[:, 1:].reshape(-1))

    def logical_state_dict(self) -> dict[str, torch.Tensor]:
        """Parameters keyed by their stable logical name."""
        return dict(self.named_parameters())

    @torch.no_grad()
    def load_logical_state(self, state: dict[str, torch.Tensor]) -> None:
        """Copy ``{name: full tensor}`` into the parameters; every name must be present."""
        own = self.logical_state_dict()
        missing = sorted(set(own) - set(state))
        if missing:
            raise KeyError(f"logical state lacks {missing}")
        for name, param in own.items():
            param.copy_(state[name].to(param.device, param.dtype))
