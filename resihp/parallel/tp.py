"""One pipeline stage executed as Megatron tensor parallelism over its TP group.

The stage owns a contiguous range of global layers (plus the embedding group on the
replica's first executable stage and the head group on its last) and holds this TP
rank's shard of every owned logical tensor, laid out in **flat buffers**:

* ``master`` FP32 parameters, ``grad`` FP32 gradient accumulators, ``exp_avg`` and
  ``exp_avg_sq`` FP32 AdamW moments -- one contiguous buffer each, so the optimizer is
  one kernel launch and a DP gradient reduction is one (bucketed) collective;
* ``work``: the compute copy of the weights -- bf16 on the B200 kernel path (refreshed
  by the fused AdamW kernel), the FP32 ``master`` itself on the reference path.

Within a layer the Q/K/V shards and the gate/up shards are adjacent, so each pair of
column-parallel projections runs as one GEMM over a fused view. Logical names map to
views into these buffers (reference: ``resihp/parallel/tp.py:113-273`` keeps one leaf
parameter per shard instead).

Two execution modes, chosen by device and dtype, over the same forward code:

* ``kernel`` (CUDA + bf16): the sm_100a ops of :mod:`resihp.ops.functional`; weight
  gradients are accumulated by the kernels straight into ``grad`` views;
* ``torch``  (CPU, or FP32): the same math in FP32 torch with autograd writing into
  ``param.grad`` (pre-bound to the ``grad`` views) -- the reference-semantics path.

Sequence parallelism (``config.sequence_parallel``) keeps the residual stream sharded
over tokens inside the TP group: column-parallel inputs are all-gathered over tokens,
row-parallel outputs reduce-scattered, and a pipeline boundary moves only token shards.
"""

from __future__ import annotations

import torch
from torch import nn
import torch.distributed as dist
from torch.nn import functional as F

from ..config import TrainConfig
from ..models.layout import TensorSpec, kernel_shape_problems, local_shape, stage_specs
from ..ops import functional as fn
from . import collectives as cc
from . import fused

_ALIGN = 64  # elements: keeps every tensor 256-byte aligned for TMA


def _numel(shape) -> int:
    n = 1
    for s in shape:
        n *= s
    return n


def local_slice(full: torch.Tensor, dim: int | None, rank: int, size: int) -> torch.Tensor:
    """This rank's contiguous shard of ``full`` (a copy)."""
    if dim is None or size == 1:
        return full.detach().clone()
    return torch.chunk(full, size, dim=dim)[rank].contiguous().clone()


REGION_FLAG_BYTES = 64 * 1024  # flag words at the head of a shared state region


class FlatState:
    """Flat FP32 master / grad / Adam buffers plus the compute copy, with named views.

    ``shared=True`` (the CUDA kernel path) places every buffer in one CUDA-IPC-exported
    region -- ``flags | master | exp_avg | exp_avg_sq | grad0 | grad1 | work`` -- so
    data-parallel peers can read each other's gradients and a post-failure reshard can
    pull state from its donors with P2P loads. The two gradient buffers alternate by
    step parity: the fused DP reduction reads the accumulated one and writes the summed
    gradient into the other, which becomes :attr:`grad` for the rest of the step.
    """

    FIELDS = ("master", "exp_avg", "exp_avg_sq", "grad0", "grad1")

    def __init__(self, entries: list[tuple[TensorSpec, tuple[int, ...]]], device, compute_dtype, *, shared=False):
        self.entries = entries
        self.offsets: dict[str, tuple[int, tuple[int, ...]]] = {}
        cursor = 0
        prev_fuse = ""
        for spec, shape in entries:
            contiguous_with_prev = spec.fuse and spec.fuse == prev_fuse
            if not contiguous_with_prev:
                cursor = (cursor + _ALIGN - 1) // _ALIGN * _ALIGN
            self.offsets[spec.name] = (cursor, shape)
            cursor += _numel(shape)
            prev_fuse = spec.fuse
        self.numel = max(1, (cursor + _ALIGN - 1) // _ALIGN * _ALIGN)
        self.step = 0
        self.shared = bool(shared)
        self.region = None
        self.handle = None
        self.field_offsets: dict[str, int] = {}
        if self.shared:
            self._alloc_region(torch.device(device), compute_dtype)
        else:
            f32 = dict(dtype=torch.float32, device=device)
            self.master = torch.zeros(self.numel, **f32)
            self.grads = (torch.zeros(self.numel, **f32),)
            self.exp_avg = torch.zeros(self.numel, **f32)
            self.exp_avg_sq = torch.zeros(self.numel, **f32)
            if compute_dtype == torch.float32:
                self.work = self.master
            else:
                self.work = torch.zeros(self.numel, dtype=compute_dtype, device=device)
        self.parity = 0
        self.grad = self.grads[0]

    def _alloc_region(self, device, compute_dtype) -> None:
        from ..ops import _ext

        n = self.numel
        work_bytes = n * torch.empty((), dtype=compute_dtype).element_size()
        off = REGION_FLAG_BYTES
        for name in self.FIELDS:
            self.field_offsets[name] = off
            off += 4 * n
        self.field_offsets["work"] = off
        total = off + work_bytes
        self.region, self.handle = _ext.require().symm_region(total, device.index or 0)
        self.region_ptr = self.region.data_ptr()

        def field(name, dtype, count):
            start = self.field_offsets[name]
            return self.region[start: start + count * torch.empty((), dtype=dtype).element_size()].view(dtype)

        self.flags = self.region[:REGION_FLAG_BYTES].view(torch.int32)
        self.master = field("master", torch.float32, n)
        self.exp_avg = field("exp_avg", torch.float32, n)
        self.exp_avg_sq = field("exp_avg_sq", torch.float32, n)
        self.grads = (field("grad0", torch.float32, n), field("grad1", torch.float32, n))
        self.work = field("work", compute_dtype, n)

    def set_parity(self, parity: int) -> None:
        self.parity = parity
        self.grad = self.grads[parity]

    def export(self) -> dict:
        """What a peer needs to read this state: IPC handle, field and tensor offsets, step."""
        return {"handle": self.handle, "fields": dict(self.field_offsets), "numel": self.numel,
                "offsets": {n: off for n, (off, _s) in self.offsets.items()}, "step": self.step}

    def view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        off, shape = self.offsets[name]
        return buf[off: off + _numel(shape)].view(shape)

    def span(self, buf: torch.Tensor, first: str, last: str, cols: int) -> torch.Tensor:
        """2-D view from ``first`` through ``last`` (adjacent tensors with ``cols`` columns)."""
        a, _ = self.offsets[first]
        b, shape = self.offsets[last]
        end = b + _numel(shape)
        return buf[a:end].view((end - a) // cols, cols)

    def refresh_work(self) -> None:
        if self.work is not self.master:
            self.work.copy_(self.master)


class TensorParallelStage:
    """This TP rank's part of one pipeline stage (see the module docstring)."""

    def __init__(
        self,
        config: TrainConfig,
        *,
        layer_ids,
        is_first: bool,
        is_last: bool,
        local_state: dict[str, torch.Tensor],
        group=None,
        device=None,
        moments: dict | None = None,
    ):
        self.config = config
        self.group = group
        self.tp_rank = 0 if group is None else dist.get_rank(group)
        self.tp_size = cc.tp_size(group)
        self.layer_ids = tuple(sorted(int(g) for g in layer_ids))
        self.is_first = bool(is_first)
        self.is_last = bool(is_last)
        self.device = torch.device("cpu") if device is None else torch.device(device)
        self.vocab_size = config.vocab_size
        self.sequence_length = config.seq_len
        self.dim = config.model_dim
        self.vocab_per_rank = config.vocab_size // self.tp_size
        self.vocab_start = self.tp_rank * self.vocab_per_rank
        self.sp = bool(config.sequence_parallel) and self.tp_size > 1
        if self.sp and config.arch == "gpt2":
            raise ValueError("sequence parallelism needs llama blocks; gpt2 blocks use all-reduce TP")
        if config.vocab_size % self.tp_size:
            raise ValueError("tp_size must divide vocab_size")
        if config.num_heads % self.tp_size or config.kv_heads % self.tp_size:
            raise ValueError("tp_size must divide the attention heads")
        self.kernel = self.device.type == "cuda" and config.dtype == "bf16"
        if config.arch == "gpt2" and self.kernel:
            raise ValueError("gpt2 blocks run on the FP32 reference path only (dtype fp32)")
        if self.kernel:
            problems = kernel_shape_problems(config, self.tp_size)
            if problems:
                raise ValueError(f"the bf16 kernels cannot run this shape at TP {self.tp_size}: " + "; ".join(problems))
        compute = torch.bfloat16 if self.kernel else torch.float32
        self.act_dtype = compute

        self.specs = stage_specs(config, self.layer_ids, self.is_first, self.is_last)
        self.spec_by_name = {s.name: s for s in self.specs}
        entries = [(s, local_shape(s, self.tp_size)) for s in self.specs]
        self.flat = FlatState(entries, self.device, compute, shared=self.kernel)
        if local_state is not None:
            with torch.no_grad():
                for s in self.specs:
                    self.flat.view(self.flat.master, s.name).copy_(local_state[s.name].to(self.device, torch.float32))
            if moments:
                self.install_moments(moments)
            self.flat.refresh_work()
        self._bind_compute_tensors()
        self.ws = None
        self.dp = None  # peer mappings of the fused DP reduction (set by the gradient reducer)
        self.hetero = None  # peer mappings of the P2P heterogeneous-replica reduction
        rows = config.micro_batch_size * config.seq_len
        if (self.kernel and fused.ENABLED and 1 < self.tp_size <= min(8, fused.MAX_DEGREE)
                and rows % self.tp_size == 0 and (rows // self.tp_size) % 128 == 0 and self.dim % 32 == 0):
            self.ws = fused.SymmetricWorkspace(group, rows // self.tp_size, self.dim, self.device)
        self.rope = None
        if config.arch == "llama":
            self.rope = fn.rope_table(config.seq_len, config.head_dim, config.rope_theta, device=self.device)

    # --- parameters -----------------------------------------------------------------

    def _bind_compute_tensors(self) -> None:
        """Compute weights (views of ``work``) and the gradient views of each grad buffer."""
        self.w: dict[str, torch.Tensor] = {}
        fused_w: dict[str, torch.Tensor] = {}
        for s in self.specs:
            if self.kernel:
                self.w[s.name] = self.flat.view(self.flat.work, s.name).detach().requires_grad_(True)
            else:
                self.w[s.name] = nn.Parameter(self.flat.view(self.flat.master, s.name))
        spans = []
        if self.config.arch == "llama":
            d = self.dim
            for gid in self.layer_ids:
                p = f"layers.{gid}."
                for key, first, last in (("qkv", "attn.q_proj.weight", "attn.v_proj.weight"),
                                         ("gate_up", "mlp.gate.weight", "mlp.up.weight")):
                    if self.kernel:
                        w = self.flat.span(self.flat.work, p + first, p + last, d).detach().requires_grad_(True)
                    else:  # a leaf of its own: autograd accumulates into the grad span set in use_grad
                        w = nn.Parameter(self.flat.span(self.flat.master, p + first, p + last, d))
                    fused_w[p + key] = w
                    spans.append((p + key, p + first, p + last))
        self._grad_sets = []
        for buf in self.flat.grads:
            g = {s.name: self.flat.view(buf, s.name) for s in self.specs}
            fw = {key: (fused_w[key], self.flat.span(buf, a, b, self.dim)) for key, a, b in spans}
            self._grad_sets.append((g, fw))
        self.use_grad(self.flat.parity)

    def use_grad(self, parity: int) -> None:
        """Make grad buffer ``parity`` the one the kernels accumulate into and ``g`` shows."""
        self.flat.set_parity(parity)
        self.g, self.fused_w = self._grad_sets[parity]
        if not self.kernel:
            for name, p in self.w.items():
                p.grad = self.g[name]
            for w, g in self.fused_w.values():
                w.grad = g

    def parameters(self):
        return list(self.w.values())

    def local_shards(self) -> dict[str, tuple[torch.Tensor, int | None]]:
        """Logical name -> (FP32 master view, shard dim)."""
        return {s.name: (self.flat.view(self.flat.master, s.name), s.shard_dim) for s in self.specs}

    def logical_state_dict(self) -> dict[str, torch.Tensor]:
        return {n: t for n, (t, _d) in self.local_shards().items()}

    def moment_views(self, name: str) -> dict[str, torch.Tensor]:
        return {
            "exp_avg": self.flat.view(self.flat.exp_avg, name),
            "exp_avg_sq": self.flat.view(self.flat.exp_avg_sq, name),
        }

    def install_moments(self, moments: dict) -> None:
        """Seed AdamW state from ``{name: {exp_avg, exp_avg_sq, step}}`` (missing names: fresh)."""
        steps = set()
        with torch.no_grad():
            for s in self.specs:
                m = moments.get(s.name)
                if not m or "exp_avg" not in m:
                    continue
                views = self.moment_views(s.name)
                views["exp_avg"].copy_(m["exp_avg"].to(self.device, torch.float32))
                views["exp_avg_sq"].copy_(m["exp_avg_sq"].to(self.device, torch.float32))
                step = m["step"]
                steps.add(int(step.item()) if torch.is_tensor(step) else int(step))
        if len(steps) > 1:
            raise ValueError(f"installed moments disagree on the AdamW step: {sorted(steps)}")
        if steps:
            self.flat.step = steps.pop()

    def zero_grad(self) -> None:
        self.flat.grad.zero_()

    def optimizer_step(self, *, grad_scale: float = 1.0) -> None:
        c = self.config
        self.flat.step += 1
        with torch.no_grad():
            fn.adamw_flat(
                self.flat.master, self.flat.grad, self.flat.exp_avg, self.flat.exp_avg_sq, self.flat.step,
                lr=c.lr, beta1=c.beta1, beta2=c.beta2, eps=c.adam_eps, weight_decay=c.weight_decay,
                p_bf16=None if self.flat.work is self.flat.master else self.flat.work, grad_scale=grad_scale,
            )

    # --- forward --------------------------------------------------------------------

    def boundary_shape(self, micro_batch_size: int) -> tuple[int, int]:
        tokens = micro_batch_size * self.sequence_length
        return (tokens // self.tp_size if self.sp else tokens, self.dim)

    def close_comm(self, *, barrier: bool = True) -> None:
        """Release the peer-memory mappings (at a safe point, with nothing in flight)."""
        if self.ws is not None:
            self.ws.close(barrier=barrier)
            self.ws = None
        if self.dp is not None:
            self.dp.close(barrier=barrier)
            self.dp = None
        if self.hetero is not None:
            self.hetero.close(barrier=barrier)
            self.hetero = None

    def _col_linear(self, h, w, g):
        """Column-parallel linear; its collective (SP: the token all-gather; otherwise the
        input gradient's all-reduce) is fused into the GEMM on the kernel path."""
        if self.ws is not None:
            return fused.ag_linear(h, w, g, self.ws) if self.sp else fused.col_linear_ar(h, w, g, self.ws)
        if self.tp_size > 1:  # the input-gradient collective overlaps the weight gradient
            return cc.column_parallel_linear(h, w, g, self.group, self.sp)
        return fn.linear(h, w, g)

    def _row_linear(self, x, w, g, residual=None):
        """Row-parallel linear (+ ``residual``); its collective (SP: the token
        reduce-scatter; otherwise the output all-reduce) is fused into the GEMM on the
        kernel path. Without TP the residual add is the GEMM's epilogue."""
        if self.ws is not None:
            y = fused.linear_rs(x, w, g, self.ws) if self.sp else fused.row_linear_ar(x, w, g, self.ws)
        elif self.tp_size == 1:
            return fn.linear(x, w, g, residual=residual)
        else:
            y = self._row_output(fn.linear(x, w, g))
        return y if residual is None else residual + y

    def _row_output(self, y):
        return cc.scatter_tokens(y, self.group) if self.sp else cc.reduce_from_tp(y, self.group)

    def _embed(self, tokens):
        ids = tokens.reshape(-1)
        w = self.w["token_embedding.weight"]
        x = fn.embedding(ids, w, self.g["token_embedding.weight"], self.vocab_start)
        if self.config.arch == "gpt2":
            x = cc.reduce_from_tp(x, self.group)
            pos = torch.arange(tokens.shape[1], device=ids.device).repeat(tokens.shape[0])
            return x + F.embedding(pos, self.w["position_embedding.weight"])
        return self._row_output(x)

    def _llama_layer(self, x, gid):
        c = self.config
        p = f"layers.{gid}."
        hq, hkv = c.num_heads // self.tp_size, c.kv_heads // self.tp_size
        # The residual stream leaves through the norm's second output, so its gradient
        # from the MLP-norm residual is summed inside the norm's backward kernel.
        h, x = fn.rmsnorm(x, self.w[p + "attn_norm.weight"], c.norm_eps, self.g[p + "attn_norm.weight"])
        wqkv, gqkv = self.fused_w[p + "qkv"]
        qkv = self._col_linear(h, wqkv, gqkv)
        o = fn.rope_attention(qkv, self.rope, c.seq_len, hq, hkv, c.head_dim)
        a = self._row_linear(o, self.w[p + "attn.o_proj.weight"], self.g[p + "attn.o_proj.weight"])
        h, x = fn.rmsnorm(a, self.w[p + "mlp_norm.weight"], c.norm_eps, self.g[p + "mlp_norm.weight"], residual=x)
        wgu, ggu = self.fused_w[p + "gate_up"]
        gu = self._col_linear(h, wgu, ggu)
        return self._row_linear(fn.swiglu(gu), self.w[p + "mlp.down.weight"], self.g[p + "mlp.down.weight"], residual=x)

    def _gpt2_layer(self, x, gid):
        p = f"layers.{gid}."
        w = self.w
        rows = x.shape[0]
        batch = rows // self.sequence_length
        heads = self.config.num_heads // self.tp_size
        hd = self.config.head_dim
        h = cc.copy_to_tp(fn.layernorm(x, w[p + "attn_norm.weight"], w[p + "attn_norm.bias"]), self.group)
        q = F.linear(h, w[p + "attn.q_proj.weight"]).view(rows, heads, hd)
        k = F.linear(h, w[p + "attn.k_proj.weight"]).view(rows, heads, hd)
        v = F.linear(h, w[p + "attn.v_proj.weight"]).view(rows, heads, hd)
        ctx = fn.causal_attention(q, k, v, batch, self.sequence_length)
        x = x + cc.reduce_from_tp(F.linear(ctx, w[p + "attn.out_proj.weight"]), self.group)
        h = cc.copy_to_tp(fn.layernorm(x, w[p + "mlp_norm.weight"], w[p + "mlp_norm.bias"]), self.group)
        m = F.linear(F.gelu(F.linear(h, w[p + "mlp.fc1.weight"])), w[p + "mlp.fc2.weight"])
        return x + cc.reduce_from_tp(m, self.group)

    def _head(self, x, tokens, loss_scale):
        c = self.config
        if c.arch == "gpt2":
            h = fn.layernorm(x, self.w["final_norm.weight"], self.w["final_norm.bias"])
        else:
            h, _ = fn.rmsnorm(x, self.w["final_norm.weight"], c.norm_eps, self.g["final_norm.weight"])
        head = "token_embedding.weight" if c.tied_embeddings else "lm_head.weight"
        if c.arch == "llama":
            logits = self._col_linear(h, self.w[head], self.g[head])
        else:
            logits = fn.linear(cc.copy_to_tp(h, self.group), self.w[head], self.g[head])
        labels = torch.full_like(tokens, -1)
        labels[:, :-1] = tokens[:, 1:]
        return fn.vocab_parallel_cross_entropy(
            logits, labels.reshape(-1), self.vocab_start, self.group if self.tp_size > 1 else None, loss_scale
        )

    def forward(self, *, tokens=None, hidden=None, loss_scale: float = 1.0):
        """Embed ``tokens`` (first stage) or continue from ``hidden``; the scaled loss on the last.

        ``loss_scale`` multiplies the summed token cross-entropy (the runtime passes
        ``1 / (tokens with a target * global micro-batch count)``).
        """
        if self.is_first:
            if tokens.shape[1] != self.sequence_length:
                raise ValueError("token sequence length does not match the stage")
            x = self._embed(tokens)
        else:
            x = hidden
        layer = self._llama_layer if self.config.arch == "llama" else self._gpt2_layer
        for gid in self.layer_ids:
            if self.config.recompute and torch.is_grad_enabled():
                x = torch.utils.checkpoint.checkpoint(layer, x, gid, use_reentrant=False)
            else:
                x = layer(x, gid)
        if not self.is_last:
            return x
        return self._head(x, tokens, loss_scale)
