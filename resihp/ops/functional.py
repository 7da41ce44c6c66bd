"""Differentiable ops of the decoder, one autograd Function per hand-written kernel.

CUDA tensors (bf16) run the sm_100a kernels; weight gradients are accumulated straight
into FP32 *main-grad* buffers passed alongside each weight (gradient-accumulation
fusion), so the bf16 weights never hold a ``.grad`` and micro-batches accumulate
without extra passes. FP32 tensors (CPU, or CUDA for a reference-semantics run on a
GPU) run the same math as plain torch expressions and let autograd fill
``param.grad``.

Conventions: activations are 2-D ``[tokens, features]``; token ``t`` of a micro-batch
is sequence ``t // S`` position ``t % S``.

Reference counterparts: the per-op torch calls of the TP stage
(``resihp/parallel/tp.py:222-273``: vocab-parallel embedding, projections, attention,
layer norms, GELU MLP, LM head) and the loss (``resihp/reference.py:41-50``).
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
from torch.autograd import Function
from torch.nn import functional as F

from . import _ext
from .gemm import linear as _gemm_linear
from .gemm import linear_dgrad, linear_wgrad


def _k():
    return _ext.require()


def on_kernels(t: torch.Tensor) -> bool:
    """bf16 CUDA tensors run the sm_100a kernels; FP32 tensors (CPU or CUDA) take the
    plain-torch FP32 reference path."""
    return t.is_cuda and t.dtype == torch.bfloat16


# ---------------------------------------------------------------------------------------
# linear
# ---------------------------------------------------------------------------------------


class _Linear(Function):
    @staticmethod
    def forward(ctx, x, w, main_grad, residual):
        ctx.save_for_backward(x, w)
        ctx.main_grad = main_grad
        ctx.has_residual = residual is not None
        return _gemm_linear(x, w, residual)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = linear_dgrad(dy, w) if ctx.needs_input_grad[0] else None
        if ctx.main_grad is not None:
            linear_wgrad(dy, x, out=ctx.main_grad, accumulate=True)
        return dx, None, None, (dy if ctx.has_residual else None)


def linear(x, w, main_grad=None, residual=None):
    """``x @ w.T`` (+ residual). CUDA: tcgen05 GEMM, wgrad accumulated into ``main_grad``."""
    if not on_kernels(x):
        y = F.linear(x, w)
        return y if residual is None else y + residual
    return _Linear.apply(x, w, main_grad, residual)


# ---------------------------------------------------------------------------------------
# RMSNorm (+ fused residual add)
# ---------------------------------------------------------------------------------------


class _RMSNorm(Function):
    @staticmethod
    def forward(ctx, x, residual, w, main_grad, eps):
        y, s, rstd = _k().rmsnorm_fwd(x, residual, w, eps)
        # An unused second output gets no gradient (None), not a materialised zero tensor.
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(s, w, rstd)
        ctx.main_grad = main_grad
        ctx.has_residual = residual is not None
        return y, s

    @staticmethod
    def backward(ctx, dy, ds_out):
        s, w, rstd = ctx.saved_tensors
        dw = ctx.main_grad if ctx.main_grad is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        dres = None if ds_out is None else ds_out.contiguous()
        if dy is None:  # only the sum output was used
            return dres, (dres if ctx.has_residual else None), None, None, None
        ds = _k().rmsnorm_bwd(dy.contiguous(), s, w, rstd, dres, dw, True)
        return ds, (ds if ctx.has_residual else None), None, None, None


def rmsnorm(x, w, eps, main_grad=None, residual=None):
    """``(rmsnorm(x + residual) * w, x + residual)``; without a residual the second output is ``x``.

    On the kernels the gradient arriving at the second output is added inside the
    backward kernel, so a stream that feeds both this norm and a later residual add
    should take the second output as that residual (one gradient sum, no extra pass).
    """
    if not on_kernels(x):
        s = x if residual is None else x + residual
        rstd = torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps)
        return s * rstd * w, s
    y, s = _RMSNorm.apply(x.contiguous(), None if residual is None else residual.contiguous(), w, main_grad, eps)
    return y, s


def layernorm(x, w, b, eps=1e-5):
    """LayerNorm of the reference GPT-2 blocks (FP32 reference path only)."""
    return F.layer_norm(x, (x.shape[-1],), w, b, eps)


# ---------------------------------------------------------------------------------------
# RoPE + causal attention (GQA)
# ---------------------------------------------------------------------------------------


def rope_table(seq: int, head_dim: int, theta: float, device=None) -> torch.Tensor:
    """``[seq, head_dim/2, 2]`` FP32 (cos, sin) of ``pos * theta^(-2i/head_dim)``."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    ang = torch.arange(seq, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.stack([ang.cos(), ang.sin()], dim=-1).to(torch.float32).contiguous().to(device)


def _rope_torch(x, cs, pos):
    """Rotate-half RoPE on ``x [T, H, D]`` with positions ``pos [T]`` (FP32 path)."""
    half = x.shape[-1] // 2
    c = cs[pos, :, 0][:, None, :]
    s = cs[pos, :, 1][:, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


class _RopeAttention(Function):
    @staticmethod
    def forward(ctx, qkv, cs, seq, hq, hkv, d):
        qkv = qkv.contiguous()
        k = _k()
        k.rope(qkv, cs, seq, hq + hkv, d, 0, False)
        scale = 1.0 / math.sqrt(d)
        out, lse = k.attn_fwd(qkv, seq, hq, hkv, d, scale)
        ctx.save_for_backward(qkv, out, lse, cs)
        ctx.dims = (seq, hq, hkv, d, scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        qkv, out, lse, cs = ctx.saved_tensors
        seq, hq, hkv, d, scale = ctx.dims
        k = _k()
        dqkv = k.attn_bwd(qkv, out, dout.contiguous(), lse, seq, hq, hkv, d, scale)
        k.rope(dqkv, cs, seq, hq + hkv, d, 0, True)
        return dqkv, None, None, None, None, None


def rope_attention(qkv, cs, seq, hq, hkv, d):
    """Causal GQA attention over the fused ``qkv [T, (hq + 2 hkv) d]``, RoPE applied to q, k.

    Returns ``[T, hq * d]``. ``cs`` is :func:`rope_table` for ``seq`` positions.
    CUDA: RoPE is applied to ``qkv`` in place (the projection output is consumed, not
    copied), so callers must not read ``qkv`` afterwards expecting un-rotated values.
    """
    if on_kernels(qkv):
        return _RopeAttention.apply(qkv, cs, seq, hq, hkv, d)
    t = qkv.shape[0]
    b = t // seq
    q, kk, v = qkv.split([hq * d, hkv * d, hkv * d], dim=-1)
    pos = torch.arange(t, device=qkv.device) % seq
    q = _rope_torch(q.reshape(t, hq, d), cs, pos)
    kk = _rope_torch(kk.reshape(t, hkv, d), cs, pos)
    v = v.reshape(t, hkv, d)
    return causal_attention(q, kk, v, b, seq)


def causal_attention(q, k, v, batch, seq):
    """Plain FP32 causal attention, ``q [T, H, D]``, ``k/v [T, Hkv, D]`` -> ``[T, H*D]``."""
    t, hq, d = q.shape
    hkv = k.shape[1]
    rep = hq // hkv
    q = q.reshape(batch, seq, hq, d).transpose(1, 2)
    k = k.reshape(batch, seq, hkv, d).transpose(1, 2).repeat_interleave(rep, dim=1)
    v = v.reshape(batch, seq, hkv, d).transpose(1, 2).repeat_interleave(rep, dim=1)
    scores = (q @ k.transpose(-2, -1)) / math.sqrt(d)
    future = torch.triu(torch.ones(seq, seq, dtype=torch.bool, device=q.device), diagonal=1)
    probs = F.softmax(scores.masked_fill(future, float("-inf")), dim=-1)
    return (probs @ v).transpose(1, 2).reshape(t, hq * d)


# ---------------------------------------------------------------------------------------
# SwiGLU
# ---------------------------------------------------------------------------------------


class _SwiGLU(Function):
    @staticmethod
    def forward(ctx, gu):
        gu = gu.contiguous()
        ctx.save_for_backward(gu)
        return _k().swiglu_fwd(gu)

    @staticmethod
    def backward(ctx, dh):
        (gu,) = ctx.saved_tensors
        return _k().swiglu_bwd(gu, dh.contiguous())


def swiglu(gu):
    """``silu(g) * u`` over the fused ``[g | u]`` projection."""
    if on_kernels(gu):
        return _SwiGLU.apply(gu)
    g, u = gu.chunk(2, dim=-1)
    return F.silu(g) * u


# ---------------------------------------------------------------------------------------
# vocab-parallel embedding
# ---------------------------------------------------------------------------------------


class _Embedding(Function):
    @staticmethod
    def forward(ctx, ids, w, main_grad, start):
        ids = ids.reshape(-1).contiguous()
        ctx.save_for_backward(ids)
        ctx.main_grad = main_grad
        ctx.start = start
        return _k().embedding_fwd(ids, w, start)

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        if ctx.main_grad is not None:
            _k().embedding_bwd(ids, dy.contiguous(), ctx.main_grad, ctx.start)
        return None, None, None, None


def embedding(ids, w, main_grad=None, start=0):
    """Rows ``ids - start`` of this rank's vocab shard ``w``; ids outside it give zeros."""
    if on_kernels(w):
        return _Embedding.apply(ids, w, main_grad, start)
    flat = ids.reshape(-1)
    local = flat - start
    outside = (local < 0) | (local >= w.shape[0])
    out = F.embedding(local.clamp(0, w.shape[0] - 1), w)
    return out.masked_fill(outside[:, None], 0.0)


# ---------------------------------------------------------------------------------------
# vocab-parallel cross-entropy
# ---------------------------------------------------------------------------------------


class _VocabParallelXent(Function):
    @staticmethod
    def forward(ctx, logits, labels, start, group, scale):
        k = _k()
        stats = k.xent_stats(logits, labels, start)
        m_loc, s_loc, z = stats[:, 0], stats[:, 1], stats[:, 2]
        if group is not None and dist.get_world_size(group) > 1:
            m = m_loc.clone()
            dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
            s = s_loc * torch.exp(m_loc - m)
            sz = torch.stack([s, z])
            dist.all_reduce(sz, group=group)
            s, z = sz[0], sz[1]
        else:
            m, s = m_loc, s_loc
        lse = (m + torch.log(s)).contiguous()
        valid = labels >= 0
        loss = ((lse - z) * valid).sum() * scale
        ctx.save_for_backward(logits, labels, lse)
        ctx.start = start
        ctx.scale = scale
        return loss

    @staticmethod
    def backward(ctx, dloss):
        logits, labels, lse = ctx.saved_tensors
        scale = (dloss.reshape(1) * ctx.scale).float().contiguous()
        _k().xent_grad(logits, labels, lse, scale, ctx.start)  # in place: logits become dlogits
        return logits, None, None, None, None


def vocab_parallel_cross_entropy(logits, labels, start=0, group=None, scale=1.0):
    """``scale * sum_t CE(t)`` over rows with a label ``>= 0``; ``logits`` is this rank's vocab shard.

    CUDA: the logits buffer is consumed (it is overwritten by its own gradient in
    backward), so callers must not reuse it.
    """
    if on_kernels(logits):
        return _VocabParallelXent.apply(logits, labels.contiguous(), start, group, scale)
    lg = logits.float()
    tp = 1 if group is None else dist.get_world_size(group)
    if tp == 1:
        valid = labels >= 0
        ce = F.cross_entropy(lg, labels.clamp_min(0), reduction="none")
        return (ce * valid).sum() * scale
    return _TorchVocabParallelXent.apply(lg, labels, start, group, scale)


class _TorchVocabParallelXent(Function):
    """The same vocab-parallel cross-entropy in plain torch (CPU / FP32 path)."""

    @staticmethod
    def forward(ctx, logits, labels, start, group, scale):
        m = logits.max(dim=-1).values
        dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
        e = torch.exp(logits - m[:, None])
        s = e.sum(-1)
        local = labels - start
        mine = (local >= 0) & (local < logits.shape[1]) & (labels >= 0)
        z = torch.where(mine, logits.gather(1, local.clamp(0, logits.shape[1] - 1)[:, None])[:, 0] - m, torch.zeros_like(m))
        sz = torch.stack([s, z])
        dist.all_reduce(sz, group=group)
        s, z = sz[0], sz[1]
        valid = labels >= 0
        loss = ((torch.log(s) - z) * valid).sum() * scale
        ctx.save_for_backward(e, s, local, mine, valid)
        ctx.scale = scale
        return loss

    @staticmethod
    def backward(ctx, dloss):
        e, s, local, mine, valid = ctx.saved_tensors
        grad = e / s[:, None]
        rows = torch.nonzero(mine)[:, 0]
        grad[rows, local[rows]] -= 1.0
        grad = grad * (valid[:, None] * (dloss * ctx.scale))
        return grad, None, None, None, None


# ---------------------------------------------------------------------------------------
# AdamW over flat buffers
# ---------------------------------------------------------------------------------------


def adamw_flat(p, g, m, v, step, *, lr, beta1, beta2, eps, weight_decay, p_bf16=None, grad_scale=1.0):
    """One AdamW step over flat FP32 buffers (torch.optim.AdamW's formulation).

    FP32 path (no bf16 copy; CPU or CUDA): the exact torch single-tensor op sequence, so
    results equal ``torch.optim.AdamW``'s single-tensor implementation bit for bit. bf16
    training path (CUDA, ``p_bf16`` given): one fused kernel that also refreshes the bf16
    working copy.
    """
    if p.is_cuda and p_bf16 is not None:  # the bf16 training path: one fused kernel
        _k().adamw(p, g, m, v, p_bf16, lr, beta1, beta2, eps, weight_decay, int(step), grad_scale)
        return
    grad = g if grad_scale == 1.0 else g * grad_scale
    p.mul_(1 - lr * weight_decay)
    m.lerp_(grad, 1 - beta1)
    v.mul_(beta2).addcmul_(grad, grad, value=1 - beta2)
    bc1 = 1 - beta1**step
    bc2 = 1 - beta2**step
    step_size = lr / bc1
    denom = (v.sqrt() / math.sqrt(bc2)).add_(eps)
    p.addcdiv_(m, denom, value=-step_size)
    if p_bf16 is not None:
        p_bf16.copy_(p)
