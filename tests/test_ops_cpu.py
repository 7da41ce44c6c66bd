"""CPU (FP32 reference-path) behaviour of the ops layer."""

import torch

from resihp.ops import functional as fn


def test_flat_adamw_is_bitwise_torch_adamw():
    torch.manual_seed(0)
    params = [torch.nn.Parameter(torch.randn(7, 5)), torch.nn.Parameter(torch.randn(11))]
    opt = torch.optim.AdamW(params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    flat_p = torch.cat([p.detach().reshape(-1) for p in params]).clone()
    m = torch.zeros_like(flat_p)
    v = torch.zeros_like(flat_p)
    for step in range(1, 6):
        grads = [torch.randn_like(p) for p in params]
        for p, g in zip(params, grads):
            p.grad = g
        opt.step()
        flat_g = torch.cat([g.reshape(-1) for g in grads])
        fn.adamw_flat(flat_p, flat_g, m, v, step, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01)
        assert torch.equal(flat_p, torch.cat([p.detach().reshape(-1) for p in params]))


def test_cpu_cross_entropy_matches_torch():
    torch.manual_seed(0)
    logits = torch.randn(10, 33, requires_grad=True)
    labels = torch.randint(0, 33, (10,))
    labels[3] = -1
    ours = fn.vocab_parallel_cross_entropy(logits, labels, scale=1 / 9)
    ref = torch.nn.functional.cross_entropy(logits, labels, ignore_index=-1)
    assert torch.allclose(ours, ref)


def test_rope_table_and_attention_shapes():
    cs = fn.rope_table(16, 8, 10000.0)
    assert cs.shape == (16, 4, 2)
    qkv = torch.randn(32, (4 + 2 * 2) * 8, requires_grad=True)
    out = fn.rope_attention(qkv, cs, 16, 4, 2, 8)
    assert out.shape == (32, 32)
    out.sum().backward()
    assert qkv.grad is not None
