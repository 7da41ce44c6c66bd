"""The whole bf16 sm_100a model against the FP32 module-form decoder (one GPU; runs last
in the GPU tier, after the per-kernel tests it builds on).

One full-batch forward + backward of the training stage on ``cuda:0`` -- every kernel
of the flagship path: embedding, RMSNorm (+residual), fused QKV / gate-up GEMMs, RoPE,
flash attention with GQA, SwiGLU, vocab cross-entropy, and their backward passes
accumulating into FP32 main-grads -- compared with :class:`resihp.model.ReferenceTransformer`,
which is plain torch (``nn.Linear``, ``nn.RMSNorm``, scaled-dot-product attention) in
FP32 on the CPU from the same initial state. bf16 operands give percent-level
differences per tensor (the attention Q/K gradients, a difference of two similar
terms, the largest); a missing, mis-routed, sign-flipped or mis-scaled gradient gives
none of the agreement asked for here (cosine >= 0.99, relative error <= 10 %).
"""

import pytest
import torch

from resihp.config import TrainConfig
from resihp.model import ReferenceTransformer
from resihp.ops import check_device_errors
from resihp.reference import ReferenceRun

pytestmark = pytest.mark.gpu

SHAPE = dict(model_dim=256, num_layers=2, batch_size=2, micro_batch_size=2, seed=0, tp=1, pp=1, dp=1,
             iterations=1, arch="llama", vocab_size=1024, seq_len=256, ffn_dim=512, init_std=0.05)


# head_dim 128 with GQA, head_dim 64 with tied embeddings: the shapes the kernel tests cover
@pytest.mark.parametrize("extra", [dict(num_heads=2, num_kv_heads=1), dict(num_heads=4, tied_embeddings=True)],
                         ids=["gqa", "tied"])
def test_bf16_model_gradients_match_the_fp32_module(extra):
    config = TrainConfig(**SHAPE, **extra, dtype="bf16")
    run = ReferenceRun(config, device="cuda:0")
    assert run.stage.kernel  # the sm_100a path, not the torch fallback
    tokens = run.batches[0]
    stage = run.stage
    start = {n: v.detach().float().cpu().clone() for n, v in stage.logical_state_dict().items()}
    stage.zero_grad()
    b, s = tokens.shape
    loss = stage.forward(tokens=tokens.cuda(), loss_scale=1.0 / (b * (s - 1)))
    loss.backward()
    torch.cuda.synchronize()
    check_device_errors(0)
    grads = {n: stage.g[n].detach().float().cpu() for n in stage.logical_state_dict()}

    module = ReferenceTransformer(TrainConfig(**SHAPE, **extra))
    for name, param in module.logical_state_dict().items():
        assert torch.equal(param.detach(), start[name]), name  # one initial model on both devices
    module.load_logical_state(start)
    want = module.loss(tokens)
    want.backward()
    assert abs(loss.item() - want.item()) <= 1e-2 * want.item(), (loss.item(), want.item())
    for name, param in module.logical_state_dict().items():
        g, ref = grads[name], param.grad
        cos = torch.nn.functional.cosine_similarity(g.flatten(), ref.flatten(), dim=0).item()
        rel = ((g - ref).norm() / ref.norm().clamp_min(1e-20)).item()
        assert cos >= 0.99 and rel <= 0.1, (name, cos, rel)


@pytest.mark.parametrize("arch", ["gpt2", "llama"])
def test_fp32_reference_runs_on_cuda_like_on_cpu(arch):
    """A reference-style FP32 config on a GPU takes the plain-torch FP32 path (the
    kernels are bf16-only) and trains like the CPU oracle (reference:
    ``tests/test_reference.py:126``, CPU vs CUDA FP32)."""
    extra = dict(ffn_dim=512, num_heads=2, init_std=0.05) if arch == "llama" else dict(num_heads=4)
    config = TrainConfig(**dict(SHAPE, **extra, arch=arch, seq_len=64, vocab_size=256, iterations=3))
    cpu, gpu = ReferenceRun(config), ReferenceRun(config, device="cuda:0")
    assert not gpu.stage.kernel
    for _ in range(3):
        a, b = cpu.step(), gpu.step()
        assert abs(a.loss - b.loss) <= 1e-4 * abs(a.loss), (a.loss, b.loss)


@pytest.mark.parametrize("arch", ["gpt2", "llama"])
def test_initial_state_does_not_depend_on_the_device(arch):
    """One seed gives one initial model whether a run trains on the CPU or a GPU (the
    CPU oracle then validates a GPU run of the same config)."""
    from resihp.models.init import DRAW_PIECE, initial_state

    extra = dict(ffn_dim=512, num_heads=2) if arch == "llama" else dict(num_heads=4)
    config = TrainConfig(**dict(SHAPE, **extra, arch=arch))
    cpu, gpu = initial_state(config), initial_state(config, device="cuda:0")
    assert cpu.keys() == gpu.keys()
    for name in cpu:
        assert gpu[name].device.type == "cuda"
        assert torch.equal(cpu[name], gpu[name].cpu()), name
    if arch == "llama":  # a tensor larger than one draw piece, drawn in pieces
        big = TrainConfig(**dict(SHAPE, **extra, arch=arch, vocab_size=DRAW_PIECE // 256 + 64))
        a = initial_state(big, names=["token_embedding.weight"])["token_embedding.weight"]
        b = initial_state(big, names=["token_embedding.weight"], device="cuda:0")["token_embedding.weight"]
        assert a.numel() > DRAW_PIECE and torch.equal(a, b.cpu())
