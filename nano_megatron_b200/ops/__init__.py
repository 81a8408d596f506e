"""Op layer: one entry point per op, CPU -> plain torch, CUDA -> our sm_100a kernels.

There is exactly one implementation per device. CPU tensors run the plain
PyTorch math in :mod:`.reference` (the correctness oracle for Gloo runs and for
the kernel tests). CUDA tensors run the hand-written kernels of the in-tree
extension ``nano_megatron_b200._C`` through :mod:`.cuda`; if that extension is
not built, the first CUDA op raises instead of silently falling back.
"""

from __future__ import annotations

import torch

from . import reference as _ref

_cuda_mod = None


def cuda_ops():
    """The CUDA op module (imports and validates the compiled extension)."""
    global _cuda_mod
    if _cuda_mod is None:
        from . import cuda as mod
        _cuda_mod = mod
    return _cuda_mod


def _impl(t: torch.Tensor):
    return cuda_ops() if t.is_cuda else _ref


def mm_nn(a, b):
    return _impl(a).mm_nn(a, b)


def mm_nt(a, b):
    return _impl(a).mm_nt(a, b)


def mm_tn_acc(a, b, out):
    return _impl(a).mm_tn_acc(a, b, out)


def rmsnorm(x, weight, eps):
    return _impl(x).rmsnorm(x, weight, eps)


def add_rmsnorm(x, a, weight, eps):
    return _impl(x).add_rmsnorm(x, a, weight, eps)


def rmsnorm_bwd(dy, x, weight, rstd, wgrad_out, dres=None):
    return _impl(x).rmsnorm_bwd(dy, x, weight, rstd, wgrad_out, dres)


def attention(qkv, batch, heads, head_dim, cos, sin):
    return _impl(qkv).attention(qkv, batch, heads, head_dim, cos, sin)


def attention_bwd(do, saved, batch, heads, head_dim, cos, sin):
    return _impl(do).attention_bwd(do, saved, batch, heads, head_dim, cos, sin)


def swiglu(gu):
    return _impl(gu).swiglu(gu)


def swiglu_bwd(da, gu):
    return _impl(gu).swiglu_bwd(da, gu)


def embedding(ids, weight, vocab_start, vocab_end):
    return _impl(weight).embedding(ids, weight, vocab_start, vocab_end)


def embedding_bwd(dy, ids, wgrad_out, vocab_start, vocab_end):
    return _impl(dy).embedding_bwd(dy, ids, wgrad_out, vocab_start, vocab_end)


def ce_local_stats(logits, target, vocab_start, vocab_end):
    return _impl(logits).ce_local_stats(logits, target, vocab_start, vocab_end)


def ce_grad(logits, target, vocab_start, gmax, gsum, scale, out_dtype):
    return _impl(logits).ce_grad(logits, target, vocab_start, gmax, gsum, scale, out_dtype)


rope_cache = _ref.rope_cache
