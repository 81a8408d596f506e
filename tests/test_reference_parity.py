"""Parity with the reference implementation itself (installed under
``baseline/_ref``, or the directory named by ``NMB_REFERENCE_PATH``; skipped
when neither holds the ``nano_megatron`` package): same seed -> identical
initial weights, logits and loss, gradients to fp32 rounding, and the same
parameters after three AdamW steps of 1F1B training."""

import os
import sys

import pytest
import torch

REF = os.environ.get("NMB_REFERENCE_PATH") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "nano_megatron")):
        pytest.skip(f"reference package not found under {REF}")
    sys.path.insert(0, REF)
    try:
        import nano_megatron.model as model
        import nano_megatron.pipeline as pipeline
        yield model, pipeline
    finally:
        sys.path.remove(REF)


def test_same_init_logits_loss_grads(ref):
    model_mod, _ = ref
    from nano_megatron_b200.models import GPT, GPTConfig
    kw = dict(vocab_size=64, n_layer=2, n_head=4, n_embd=32, seq_len=8)
    torch.manual_seed(0)
    r = model_mod.GPT(model_mod.GPTConfig(**kw))
    torch.manual_seed(0)
    m = GPT(GPTConfig(**kw))
    for (n1, p1), (n2, p2) in zip(r.named_parameters(), m.named_parameters(), strict=True):
        assert n1 == n2 and torch.equal(p1, p2)
    x, y = torch.randint(0, 64, (2, 8)), torch.randint(0, 64, (2, 8))
    torch.testing.assert_close(m(x), r(x), rtol=0, atol=0)
    lr, lm = r(x, y), m(x, y)
    torch.testing.assert_close(lm, lr, rtol=1e-6, atol=1e-6)
    lr.backward()
    lm.backward()
    for (n, p1), (_, p2) in zip(r.named_parameters(), m.named_parameters(), strict=True):
        torch.testing.assert_close(p2.grad, p1.grad, rtol=1e-5, atol=1e-7, msg=n)


def test_training_steps_match(ref):
    model_mod, pipeline = ref
    from nano_megatron_b200 import GPT, GPTConfig, ParallelContext, forward_backward_1f1b
    from nano_megatron_b200.optim import FusedAdamW
    from nano_megatron_b200.utils.data import synthetic_batches
    kw = dict(vocab_size=64, n_layer=2, n_head=4, n_embd=32, seq_len=8)
    cfg = GPTConfig(**kw)
    torch.manual_seed(0)
    r = model_mod.GPT(model_mod.GPTConfig(**kw))
    torch.manual_seed(0)
    m = GPT(cfg)
    o1, o2 = torch.optim.AdamW(r.parameters(), lr=1e-3), FusedAdamW(m, lr=1e-3)
    ctx = ParallelContext.single()
    for step in range(3):
        o1.zero_grad(set_to_none=True)
        o2.zero_grad()
        batches = synthetic_batches(cfg, 2, 2, step)
        l1 = pipeline.forward_backward_1f1b(r, batches, cfg, "cpu", ctx)
        l2 = forward_backward_1f1b(m, batches, cfg, "cpu", ctx)
        o1.step()
        o2.step()
        torch.testing.assert_close(sum(l2), sum(l1), rtol=1e-5, atol=1e-6)
    for p1, p2 in zip(r.parameters(), m.parameters(), strict=True):
        torch.testing.assert_close(p2, p1, rtol=1e-4, atol=1e-5)


def test_state_dicts_load_both_ways(ref):
    """A reference model's state dict loads into this model with strict key and
    shape checks, and the other way round; the loaded models agree."""
    model_mod, _ = ref
    from nano_megatron_b200.models import GPT, GPTConfig
    kw = dict(vocab_size=64, n_layer=2, n_head=4, n_embd=32, seq_len=8)
    torch.manual_seed(1)
    r = model_mod.GPT(model_mod.GPTConfig(**kw))
    torch.manual_seed(2)
    m = GPT(GPTConfig(**kw))
    m.load_state_dict(r.state_dict(), strict=True)
    x = torch.randint(0, 64, (2, 8))
    torch.testing.assert_close(m(x), r(x), rtol=0, atol=0)
    torch.manual_seed(3)
    m2 = GPT(GPTConfig(**kw))
    r.load_state_dict(m2.state_dict(), strict=True)
    torch.testing.assert_close(r(x), m2(x), rtol=0, atol=0)
