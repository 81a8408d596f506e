"""Whole-block recompute: identical results, training only; bf16 compute path."""

from dataclasses import replace

import torch

from nano_megatron_b200.models import GPT, GPTConfig


def test_recompute_matches_normal():
    cfg = GPTConfig(vocab_size=64, n_layer=2, n_head=4, n_embd=32, seq_len=8)
    x = torch.randint(0, 64, (2, 8))
    y = torch.randint(0, 64, (2, 8))
    torch.manual_seed(0)
    a = GPT(cfg)
    b = GPT(replace(cfg, recompute=True))
    b.load_state_dict(a.state_dict())
    torch.testing.assert_close(b(x), a(x))
    la, lb = a(x, y), b(x, y)
    la.backward()
    lb.backward()
    torch.testing.assert_close(lb, la)
    for (n, pa), (_, pb) in zip(a.named_parameters(), b.named_parameters()):
        torch.testing.assert_close(pb.grad, pa.grad, msg=n)


def test_recompute_only_in_training(monkeypatch):
    cfg = GPTConfig(vocab_size=64, n_layer=2, n_head=4, n_embd=32, seq_len=8, recompute=True)
    calls = 0

    def counting(fn, *args, **kwargs):
        nonlocal calls
        calls += 1
        return fn(*args)

    monkeypatch.setattr("nano_megatron_b200.models.gpt.checkpoint", counting)
    x = torch.randint(0, 64, (2, 8))
    m = GPT(cfg)
    m(x)
    assert calls == cfg.n_layer
    m.eval()
    m(x)
    assert calls == cfg.n_layer


def test_bf16_compute_finite():
    cfg = GPTConfig(vocab_size=64, n_layer=2, n_head=4, n_embd=32, seq_len=8, compute_dtype="bfloat16")
    m = GPT(cfg)
    x = torch.randint(0, 64, (2, 8))
    y = torch.randint(0, 64, (2, 8))
    assert m(x).dtype == torch.bfloat16
    loss = m(x, y)
    loss.backward()
    assert loss.dtype == torch.float32 and torch.isfinite(loss)
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in m.parameters())


def test_extensions_ffn_theta_untied():
    cfg = GPTConfig(vocab_size=64, n_layer=2, n_head=4, n_embd=32, seq_len=8, ffn_hidden_size=40,
                    rope_theta=500000.0, tie_word_embeddings=False)
    m = GPT(cfg)
    assert m.layers[0].mlp.gate.weight.shape == (32, 40)
    assert m.lm_head.weight is not m.embedding.weight
    from nano_megatron_b200.ops.reference import rope_cache
    cos, _ = rope_cache(8, 8, 500000.0)
    torch.testing.assert_close(m.rope_cos, cos)
    loss = m(torch.randint(0, 64, (2, 8)), torch.randint(0, 64, (2, 8)))
    loss.backward()
    assert m.lm_head.weight.grad.abs().sum() > 0 and m.embedding.weight.grad.abs().sum() > 0
    assert cfg.num_parameters() == sum(p.numel() for p in m.parameters())
