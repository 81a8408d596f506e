"""The whole GPT stage on the GPU (bf16, our kernels) against the same model
on the CPU in fp32 (plain torch math) from identical weights: loss, logits and
every gradient within bf16 tolerance; recomputation reproduces the gradients
of the plain forward bit for bit (the first forward of a recomputed layer
skips the tensors only a backward reads); and AdamW steps through the fused
kernel."""

import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from nano_megatron_b200 import GPT, GPTConfig, ParallelContext, forward_backward_1f1b  # noqa: E402
from nano_megatron_b200.optim import FusedAdamW  # noqa: E402
from nano_megatron_b200.utils.data import synthetic_batches  # noqa: E402

DEV = torch.device("cuda", 0)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("recompute,tie", [(False, True), (True, False)])
def test_gpt_cuda_matches_cpu(recompute, tie):
    cfg = GPTConfig(vocab_size=512, n_layer=2, n_head=2, n_embd=256, seq_len=128, ffn_hidden_size=512,
                    compute_dtype="bfloat16", recompute=recompute, tie_word_embeddings=tie, rope_theta=500000.0,
                    init_std=0.08)  # large enough that attention is far from uniform
    torch.manual_seed(0)
    cpu = GPT(dataclasses.replace(cfg, compute_dtype="float32"))  # fp32 oracle
    gpu = GPT(cfg)
    gpu.load_state_dict(cpu.state_dict())
    gpu = gpu.to(DEV)
    x = torch.randint(0, 512, (2, 128))
    y = torch.randint(0, 512, (2, 128))
    loss_c = cpu(x, y)
    loss_c.backward()
    loss_g = gpu(x.to(DEV), y.to(DEV))
    loss_g.backward()
    assert abs(loss_g.item() - loss_c.item()) < 2e-2 * abs(loss_c.item())
    for (n, pc), (_, pg) in zip(cpu.named_parameters(), gpu.named_parameters()):
        assert _rel(pg.grad.cpu(), pc.grad) < 6e-2, (n, _rel(pg.grad.cpu(), pc.grad))
    with torch.no_grad():
        assert _rel(gpu(x.to(DEV)).cpu(), cpu(x)) < 2e-2


def test_recompute_gives_identical_gradients():
    cfg = GPTConfig(vocab_size=512, n_layer=3, n_head=2, n_embd=256, seq_len=256, ffn_hidden_size=704,
                    compute_dtype="bfloat16", tie_word_embeddings=False, init_std=0.05)
    x = torch.randint(0, 512, (2, 256), device=DEV)
    y = torch.randint(0, 512, (2, 256), device=DEV)
    grads, losses = {}, {}
    for recompute in (False, True):
        torch.manual_seed(0)
        model = GPT(dataclasses.replace(cfg, recompute=recompute), device=DEV)
        loss = model(x, y)
        loss.backward()
        losses[recompute] = loss.item()
        grads[recompute] = [p.grad.clone() for p in model.parameters()]
    assert losses[True] == losses[False]
    for g0, g1 in zip(grads[False], grads[True]):
        assert torch.equal(g0, g1)


def test_training_step_on_gpu_decreases_loss():
    cfg = GPTConfig(vocab_size=256, n_layer=2, n_head=2, n_embd=256, seq_len=128, compute_dtype="bfloat16")
    torch.manual_seed(0)
    model = GPT(cfg, device=DEV)
    opt = FusedAdamW(model, lr=3e-3)
    batches = [(x.to(DEV), x.to(DEV)) for x, _ in synthetic_batches(cfg, 2, 2, 0)]
    losses = []
    for _ in range(8):
        opt.zero_grad()
        losses.append(sum(forward_backward_1f1b(model, batches, cfg, DEV, ParallelContext.single())).item())
        opt.step()
    assert losses[-1] < losses[0] - 0.5, losses


def test_gpt_cuda_fp32_matches_cpu_tightly():
    """fp32 mode on CUDA (exact-fp32 kernels) reproduces the CPU model to the
    distributed tests' tolerance."""
    cfg = GPTConfig(vocab_size=128, n_layer=2, n_head=4, n_embd=64, seq_len=32, init_std=0.05)
    torch.manual_seed(0)
    cpu = GPT(cfg)
    gpu = GPT(cfg)
    gpu.load_state_dict(cpu.state_dict())
    gpu = gpu.to(DEV)
    x = torch.randint(0, 128, (2, 32))
    y = torch.randint(0, 128, (2, 32))
    lc = cpu(x, y)
    lc.backward()
    lg = gpu(x.to(DEV), y.to(DEV))
    lg.backward()
    torch.testing.assert_close(lg.cpu(), lc, rtol=1e-5, atol=1e-5)
    for (n, pc), (_, pg) in zip(cpu.named_parameters(), gpu.named_parameters()):
        torch.testing.assert_close(pg.grad.cpu(), pc.grad, rtol=1e-4, atol=1e-5, msg=n)
