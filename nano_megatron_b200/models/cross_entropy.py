"""Cross entropy over vocabulary-sharded logits, without gathering the logits.

Each rank reduces its ``[T, V/tp]`` shard to three per-token numbers (local
max, sum of ``exp(logit - local max)``, target logit if the target is in this
shard), the TP group exchanges only those (one all-gather of ``[3, T]``), and
every rank merges them into the global max, sum and target logit. Traffic is
O(tokens), not O(tokens * vocab). The model's LM head uses the fused version
of the same computation (``functional.lm_head_cross_entropy``); this function
is the standalone form for logits a caller already has.

Parity: ``nano_megatron/cross_entropy.py:16-85`` (same loss and gradient,
mean over tokens, fp32 math).
"""

from __future__ import annotations

import torch

from .. import ops
from ..parallel.context import ParallelContext
from .functional import merge_ce_stats


class _VocabParallelCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, target, vocab_start, vocab_end, pctx):
        flat = logits.reshape(-1, logits.shape[-1]).float()
        tgt = target.reshape(-1)
        mx, se, tl, _ = ops.ce_local_stats(flat, tgt, vocab_start, vocab_end)
        gm, gs, gt = merge_ce_stats(mx, se, tl, pctx)
        ctx.save_for_backward(flat, tgt, gm, gs)
        ctx.vocab_start, ctx.shape = vocab_start, logits.shape
        return (gs.log() + gm - gt).view(target.shape)

    @staticmethod
    def backward(ctx, grad):
        flat, tgt, gm, gs = ctx.saved_tensors
        d = ops.ce_grad(flat, tgt, ctx.vocab_start, gm, gs, grad.reshape(-1).float(), torch.float32)
        return d.view(ctx.shape), None, None, None, None


def vocab_parallel_cross_entropy(logits: torch.Tensor, target: torch.Tensor, vocab_start: int,
                                 vocab_end: int, ctx: ParallelContext) -> torch.Tensor:
    """Mean cross entropy of ``logits [..., V/tp]`` against global ids ``target [...]``."""
    vocab_size = ctx.tp_size * (vocab_end - vocab_start)
    if not target.is_cuda and (torch.any(target < 0) or torch.any(target >= vocab_size)):
        raise ValueError("target token id is outside the model vocabulary")
    return _VocabParallelCE.apply(logits, target, vocab_start, vocab_end, ctx).mean()
