"""The standalone ``apply_rope`` (reference ``model.py:84-89`` layout:
``[b, heads, s, head_dim]``) against rotary embedding written as complex
multiplication: the halves ``(a, b)`` form ``a + i b``, rotated by ``e^{i p w}``."""

import torch

from nano_megatron_b200.models import apply_rope, build_rope_cache


def _complex_rope(x, theta):
    s, d = x.shape[-2], x.shape[-1]
    w = theta ** (-torch.arange(0, d, 2, dtype=torch.float64) / d)
    angle = torch.arange(s, dtype=torch.float64)[:, None] * w[None, :]
    z = torch.complex(x[..., : d // 2].double(), x[..., d // 2:].double()) * torch.polar(torch.ones_like(angle), angle)
    return torch.cat([z.real, z.imag], dim=-1)


def test_apply_rope_matches_complex_rotation():
    torch.manual_seed(3)
    x = torch.randn(2, 3, 40, 64)
    cos, sin = build_rope_cache(64, 64, "cpu", base=500000.0)  # tables longer than the sequence
    y = apply_rope(x, cos, sin)
    assert y.shape == x.shape and y.dtype == torch.float32
    torch.testing.assert_close(y.double(), _complex_rope(x, 500000.0), rtol=1e-5, atol=1e-5)


def test_apply_rope_inverse_and_norm():
    torch.manual_seed(4)
    x = torch.randn(1, 2, 16, 32)
    cos, sin = build_rope_cache(16, 32, "cpu")
    y = apply_rope(x, cos, sin)
    # a rotation keeps each (a, b) pair's length, and the opposite angle undoes it
    pair = lambda t: t[..., :16] ** 2 + t[..., 16:] ** 2  # noqa: E731
    torch.testing.assert_close(pair(y), pair(x), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(apply_rope(y, cos, -sin), x, rtol=1e-5, atol=1e-5)
    # bf16 input with fp32 tables promotes like the reference's expression
    assert apply_rope(x.bfloat16(), cos, sin).dtype == torch.float32
