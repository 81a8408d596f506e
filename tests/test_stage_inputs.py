"""What a stage's forward accepts and exposes: a non-first pipeline stage takes
its hidden state batch-first ``[b, s, H]``, as the reference's stages do, and
refuses any other layout with the expected shape (instead of reading swapped
axes); a non-last stage returns the same layout; forward hooks on the model's
modules fire."""

import pytest
import torch

from nano_megatron_b200 import GPT, GPTConfig, ParallelContext


def _last_stage(**kw):
    ctx = ParallelContext(rank=1, world_size=2, tp_size=1, tp_rank=0, pp_size=2, pp_rank=1,
                          dp_size=1, dp_rank=0, pp_ranks=(0, 1))
    cfg = GPTConfig(vocab_size=64, n_layer=2, n_head=4, n_embd=32, seq_len=8, **kw)
    torch.manual_seed(0)
    return GPT(cfg, ctx), cfg


def test_batch_first_hidden_state_is_accepted():
    model, cfg = _last_stage()
    h = torch.randn(3, cfg.seq_len, cfg.n_embd)
    labels = torch.randint(0, cfg.vocab_size, (3, cfg.seq_len))
    loss = model(h, labels)
    assert loss.ndim == 0 and torch.isfinite(loss)
    logits = model(h)
    assert logits.shape == (3, cfg.seq_len, cfg.vocab_size)


@pytest.mark.parametrize("shape", [(8, 3, 32), (3, 8, 16), (24, 32)])
def test_other_layouts_are_refused(shape):
    model, _ = _last_stage()
    with pytest.raises(ValueError, match=r"batch-first \[batch, 8, 32\]"):
        model(torch.randn(*shape))


def test_a_middle_stage_returns_batch_first():
    ctx = ParallelContext(rank=1, world_size=3, tp_size=1, tp_rank=0, pp_size=3, pp_rank=1,
                          dp_size=1, dp_rank=0, pp_ranks=(0, 1, 2))
    torch.manual_seed(0)
    model = GPT(GPTConfig(vocab_size=64, n_layer=3, n_head=4, n_embd=32, seq_len=8), ctx)
    h = torch.randn(3, 8, 32)
    out = model(h)
    assert out.shape == (3, 8, 32)
    # each sequence of the microbatch is processed on its own (causal attention within it)
    torch.testing.assert_close(model(h[1:2])[0], out[1], rtol=1e-5, atol=1e-6)


def test_forward_hooks_on_the_model_modules_fire():
    """The model calls its modules (row form), so hooks registered on them run,
    as they do on the reference's modules."""
    torch.manual_seed(0)
    cfg = GPTConfig(vocab_size=64, n_layer=2, n_head=4, n_embd=32, seq_len=8)
    model = GPT(cfg, ParallelContext.single())
    seen = []
    modules = [model.embedding, *model.layers, model.layers[0].attn, model.layers[0].mlp, model.final_norm]
    for m in modules:
        m.register_forward_hook(lambda mod, _i, out, seen=seen: seen.append((type(mod).__name__, tuple(out.shape))))
    model(torch.randint(0, 64, (3, 8)), torch.randint(0, 64, (3, 8)))
    names = [n for n, _ in seen]
    assert names.count("TransformerLayer") == 2 and "VocabParallelEmbedding" in names
    assert "ParallelAttention" in names and "ParallelMLP" in names and "RMSNorm" in names
    assert all(shape == (8 * 3, 32) for _, shape in seen)
