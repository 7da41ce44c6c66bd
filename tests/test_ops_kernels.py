"""Numerics of the non-GEMM sm_100a kernels against FP32 torch references of the same op."""

import math

import pytest
import torch

from resihp.ops import functional as fn

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("d", [128, 256, 1024, 2048, 5120])
@pytest.mark.parametrize("with_residual", [False, True])
def test_rmsnorm(d, with_residual):
    torch.manual_seed(0)
    rows = 333
    x = torch.randn(rows, d, device="cuda").bfloat16().requires_grad_()
    r = torch.randn(rows, d, device="cuda").bfloat16().requires_grad_() if with_residual else None
    w = (1 + 0.1 * torch.randn(d, device="cuda")).bfloat16().requires_grad_()
    mg = torch.zeros(d, device="cuda")
    y, s = fn.rmsnorm(x, w, 1e-5, main_grad=mg, residual=r)
    # fp32 reference
    xf = x.detach().float().requires_grad_()
    rf = r.detach().float().requires_grad_() if with_residual else None
    wf = w.detach().float().requires_grad_()
    sf = xf if rf is None else xf + rf
    sf_r = sf.bfloat16().float() if with_residual else sf
    yf = sf_r * torch.rsqrt(sf_r.pow(2).mean(-1, keepdim=True) + 1e-5) * wf
    assert _rel(y, yf) < 1e-2
    dy = torch.randn_like(y)
    ds = torch.randn_like(s) if with_residual else None
    (y.float() * dy.float()).sum().backward(retain_graph=True) if ds is None else torch.autograd.backward([y, s], [dy, ds])
    ref_out = (yf * dy.float()).sum() + ((sf * ds.float()).sum() if ds is not None else 0)
    ref_out.backward()
    assert _rel(x.grad, xf.grad) < 2e-2
    if with_residual:
        assert _rel(r.grad, rf.grad) < 2e-2
    assert _rel(mg, wf.grad) < 1e-2


@pytest.mark.parametrize("f", [704, 6])  # 16-byte vector kernels; scalar kernels (f % 8 != 0)
def test_swiglu(f):
    torch.manual_seed(0)
    gu = torch.randn(300, 2 * f, device="cuda").bfloat16().requires_grad_()
    h = fn.swiglu(gu)
    gf = gu.detach().float().requires_grad_()
    g, u = gf.chunk(2, -1)
    hf = torch.nn.functional.silu(g) * u
    assert _rel(h, hf) < 1e-2
    dh = torch.randn_like(h)
    h.backward(dh)
    hf.backward(dh.float())
    assert _rel(gu.grad, gf.grad) < 1e-2


@pytest.mark.parametrize("hq,hkv,d,seq,batch", [(4, 4, 64, 256, 2), (8, 2, 128, 384, 1), (16, 16, 128, 2048, 1)])
def test_rope_attention(hq, hkv, d, seq, batch):
    torch.manual_seed(0)
    t = batch * seq
    cs = fn.rope_table(seq, d, 10000.0, device="cuda")
    qkv = (torch.randn(t, (hq + 2 * hkv) * d, device="cuda")).bfloat16().requires_grad_()
    qf = qkv.detach().float().cpu().requires_grad_()  # before: the CUDA op rotates its input in place
    out = fn.rope_attention(qkv, cs, seq, hq, hkv, d)
    ref = fn.rope_attention(qf, cs.cpu(), seq, hq, hkv, d)
    assert _rel(out.cpu(), ref) < 2e-2
    dout = torch.randn_like(out)
    out.backward(dout)
    ref.backward(dout.float().cpu())
    assert _rel(qkv.grad.cpu(), qf.grad) < 3e-2
    from resihp.ops import check_device_errors
    check_device_errors()


def test_embedding_vocab_parallel():
    torch.manual_seed(0)
    v, d, start = 64, 256, 32
    w = torch.randn(v, d, device="cuda").bfloat16().requires_grad_()
    ids = torch.randint(0, 128, (2, 100), device="cuda")
    mg = torch.zeros(v, d, device="cuda")
    out = fn.embedding(ids, w, mg, start)
    ref = fn.embedding(ids.cpu(), w.detach().float().cpu(), None, start)
    assert torch.equal(out.float().cpu(), ref)
    dy = torch.randn_like(out)
    out.backward(dy)
    wf = w.detach().float().cpu().requires_grad_()
    fn.embedding(ids.cpu(), wf, None, start).backward(dy.float().cpu())
    assert _rel(mg.cpu(), wf.grad) < 1e-5


def test_cross_entropy():
    torch.manual_seed(0)
    rows, v = 257, 32000
    logits = (3 * torch.randn(rows, v, device="cuda")).bfloat16()
    labels = torch.randint(0, v, (rows,), device="cuda")
    labels[-3:] = -1
    ref_l = logits.detach().float().cpu().requires_grad_()
    loss = fn.vocab_parallel_cross_entropy(logits.clone().requires_grad_(), labels, scale=1 / 254)
    ref = fn.vocab_parallel_cross_entropy(ref_l, labels.cpu(), scale=1 / 254)
    assert abs(loss.item() - ref.item()) < 1e-3 * abs(ref.item())
    lg = logits.clone().requires_grad_()
    loss = fn.vocab_parallel_cross_entropy(lg, labels, scale=1 / 254)
    loss.backward()
    ref.backward()
    assert _rel(lg.grad.cpu(), ref_l.grad) < 2e-2


@pytest.mark.parametrize("n", [100_003, 100_000])  # scalar kernel; four-wide kernel
def test_adamw_flat_matches_cpu(n):
    torch.manual_seed(0)
    p = torch.randn(n)
    g = torch.randn(n)
    m = torch.zeros(n)
    v = torch.zeros(n)
    pc, mc, vc = p.clone(), m.clone(), v.clone()
    pd, gd, md, vd = p.cuda(), g.cuda(), m.cuda(), v.cuda()
    pb = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    hp = dict(lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1)
    for step in (1, 2, 3):
        fn.adamw_flat(pc, g, mc, vc, step, **hp)
        fn.adamw_flat(pd, gd, md, vd, step, p_bf16=pb, **hp)
    assert torch.allclose(pd.cpu(), pc, rtol=1e-6, atol=1e-7)
    assert torch.allclose(pb.float().cpu(), pc, rtol=1e-2)
