"""``cuda_shape_problems``: the shapes the CUDA kernels take, checked once on
the model's first CUDA forward so a misfit fails with an actionable message
rather than inside a kernel binding."""

from types import SimpleNamespace

from nano_megatron_b200.models import GPTConfig, cuda_shape_problems


def ctx(tp):
    return SimpleNamespace(tp_size=tp)


def test_named_configs_fit():
    llama8b = GPTConfig(vocab_size=128256, n_layer=32, n_head=32, n_embd=4096, seq_len=8192, ffn_hidden_size=14336)
    assert cuda_shape_problems(llama8b, ctx(1)) == [] and cuda_shape_problems(llama8b, ctx(4)) == []
    c13b = GPTConfig(vocab_size=32000, n_layer=24, n_head=16, n_embd=2048, seq_len=2048, ffn_hidden_size=5632)
    assert cuda_shape_problems(c13b, ctx(8)) == []
    tiny = GPTConfig(vocab_size=1024, n_layer=4, n_head=8, n_embd=256, seq_len=128, ffn_hidden_size=688)
    assert cuda_shape_problems(tiny, ctx(2)) == []  # head size 32 runs the materialized attention
    assert cuda_shape_problems(GPTConfig(), ctx(1)) == []  # the reference CLI's defaults


def test_misfits_are_named():
    gpt2 = GPTConfig(vocab_size=50257, n_layer=12, n_head=12, n_embd=768, seq_len=1024)
    (msg,) = cuda_shape_problems(gpt2, ctx(1))
    assert "vocabulary" in msg and "50264" in msg
    assert any("pad vocab_size to 50272" in m for m in cuda_shape_problems(
        GPTConfig(vocab_size=50257, n_layer=12, n_head=12, n_embd=768, seq_len=1024), ctx(4)))
    odd_head = GPTConfig(vocab_size=256, n_head=4, n_embd=40, seq_len=32)
    msgs = cuda_shape_problems(odd_head, ctx(1))
    assert any("head_dim 10" in m for m in msgs)
    wide = GPTConfig(vocab_size=256, n_head=128, n_embd=16384, seq_len=32)
    assert any("8192" in m for m in cuda_shape_problems(wide, ctx(1)))
    odd_ffn = GPTConfig(vocab_size=256, n_head=2, n_embd=256, seq_len=32, ffn_hidden_size=100)
    assert any("SwiGLU width" in m for m in cuda_shape_problems(odd_ffn, ctx(1)))
