"""Autograd functions of the model: linear layers with their TP collectives,
RMSNorm, attention, SwiGLU, embedding and the fused LM-head cross entropy.

Weight gradients are accumulated straight into each parameter's fp32
``main_grad`` (a view into the stage's flat gradient buffer) inside the
backward, instead of being returned to autograd; this is what lets the
optimizer, the norm and the data-parallel reduction work on one flat buffer.
A weight without ``main_grad`` (a standalone layer) gets its gradient through
autograd as usual.

Collectives: each function names its communication ``mode``.

* column linear: ``"f"`` (identity fwd, all-reduce bwd), ``"ag"`` (sequence
  all-gather fwd, reduce-scatter bwd) or ``"none"``;
* row linear: ``"g"`` (all-reduce fwd), ``"rs"`` (reduce-scatter fwd,
  all-gather bwd) or ``"none"``.

On CUDA with a TP group of more than one GPU, ``"ag"`` and ``"rs"`` run the
fused all-gather->GEMM and GEMM->reduce-scatter kernels of
:mod:`nano_megatron_b200.ops.fused_tp`; everywhere else they run the generic
collectives of :mod:`nano_megatron_b200.parallel.mappings`.

Parity: ``nano_megatron/tp_layers.py:34-132``, ``model.py:65-192`` and
``cross_entropy.py:16-85`` (same values; the collectives are the adjoint pairs
of ``mappings.py:83-134``).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from ..parallel import mappings as M
from ..parallel.context import ParallelContext


# Observer of gradient writes: called with each ``main_grad`` tensor right
# after a backward enqueued the kernel that accumulates into it (the
# data-parallel bucketer of :mod:`nano_megatron_b200.parallel.grads` listens).
_grad_observer = None


def set_grad_observer(fn):
    """Install ``fn(main_grad)`` as the gradient-write observer; returns the previous one."""
    global _grad_observer
    previous, _grad_observer = _grad_observer, fn
    return previous


def _grad_written(tensor) -> None:
    if _grad_observer is not None:
        _grad_observer(tensor)


# True while a checkpointed layer runs its first forward: torch.utils.checkpoint
# drops what that forward saves and recomputes the layer before its backward,
# so an op may skip materializing tensors that exist only to be saved.
_discarded_forward = [False]


class discarded_forward:
    """Context manager marking (or not) the first forward of a recomputed layer."""

    def __init__(self, active: bool):
        self.active = active

    def __enter__(self):
        self.previous, _discarded_forward[0] = _discarded_forward[0], self.active

    def __exit__(self, *exc):
        _discarded_forward[0] = self.previous


def _placeholder(shape, like: torch.Tensor) -> torch.Tensor:
    """A tensor with the metadata checkpointing compares (shape, dtype, device) and no storage of that size."""
    return torch.empty((1,) * len(shape), dtype=like.dtype, device=like.device).expand(*shape)


class WeightRef:
    """A weight as the kernels see it: master data, compute copy, grad buffer.

    ``data`` is the fp32 master (a Parameter or a region of the flat buffer
    that several Parameters view), ``compute`` an optional persistent bf16
    mirror kept in sync by the optimizer, ``main_grad`` the fp32 gradient
    accumulator (None for standalone layers), ``params`` the Parameters that
    ``data`` backs, in order.
    """

    __slots__ = ("data", "compute", "main_grad", "params")

    def __init__(self, data, params, compute=None, main_grad=None):
        self.data = data
        self.params = tuple(params)
        self.compute = compute
        self.main_grad = main_grad

    @classmethod
    def of(cls, param: torch.nn.Parameter) -> "WeightRef":
        return cls(param, (param,), getattr(param, "compute_copy", None),
                   getattr(param, "main_grad", None))

    def for_compute(self, dtype: torch.dtype) -> torch.Tensor:
        if self.compute is not None and self.compute.dtype == dtype:
            return self.compute
        data = self.data.detach()
        return data if data.dtype == dtype else data.to(dtype)

    def accumulate(self, grad_fn, *args):
        """Accumulate via ``grad_fn(*args, out)``; returns autograd grads for ``params``."""
        if self.main_grad is not None:
            grad_fn(*args, self.main_grad)
            _grad_written(self.main_grad)
            return (None,) * len(self.params)
        if len(self.params) != 1:
            raise RuntimeError("a fused weight needs a main_grad buffer")
        out = torch.zeros(self.data.shape, dtype=torch.float32, device=self.data.device)
        grad_fn(*args, out)
        return (out.to(self.data.dtype),)


# ---------------------------------------------------------------- comm glue
def _use_fused(pctx: ParallelContext, x: torch.Tensor, rows_local: int) -> bool:
    """Fused all-gather/reduce-scatter GEMM kernels: CUDA, bf16, TP > 1, enabled."""
    if not (x.is_cuda and x.dtype == torch.bfloat16 and pctx.tp_size > 1
            and pctx.resources.get("fused_tp", False)):
        return False
    from ..ops import fused_tp
    return fused_tp.supported(rows_local, pctx)


def _use_fused_ce(pctx: ParallelContext, x: torch.Tensor, w: torch.Tensor, mode: str) -> bool:
    """Fused LM-head + cross-entropy kernels: CUDA, bf16; across GPUs only when enabled."""
    if not (x.is_cuda and x.dtype == torch.bfloat16):
        return False
    from ..ops import fused_tp
    if not fused_tp.ce_supported(x.shape[0], w.shape[0]):
        return False
    return pctx.tp_size == 1 or (pctx.tp_size <= 8 and pctx.resources.get("fused_tp", False))


def _ag(x, pctx):
    return M.all_gather_sequence(x, pctx.tp_group, pctx.tp_size)


def _rs(x, pctx):
    return M.reduce_scatter_sequence(x, pctx.tp_group, pctx.tp_size)


def _ar(x, pctx):
    return M._all_reduce(x.contiguous(), pctx.tp_group, pctx.tp_size)


# ------------------------------------------------------------ column linear
class _ColumnLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, wref, pctx, mode, dtype, *params):
        x = x if x.dtype == dtype else x.to(dtype)
        w = wref.for_compute(dtype)
        ctx.gathered = mode == "ag" and _use_fused(pctx, x, x.shape[0])
        if ctx.gathered:
            # The kernel also leaves a private copy of AG(x) for the weight
            # gradient, so the backward needs no second all-gather (not in the
            # first forward of a recomputed layer, whose saves are dropped).
            from ..ops import fused_tp
            if _discarded_forward[0]:
                y = fused_tp.all_gather_matmul(x, w, pctx)
                X = _placeholder((y.shape[0], x.shape[1]), x)
            else:
                X, y = fused_tp.all_gather_matmul(x, w, pctx, save_gathered=True)
            ctx.save_for_backward(X, w)
        else:
            X = _ag(x, pctx) if mode == "ag" else x
            y = ops.mm_nn(X, w)
            ctx.save_for_backward(x, w)
        ctx.wref, ctx.pctx, ctx.mode = wref, pctx, mode
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        pctx, mode, wref = ctx.pctx, ctx.mode, ctx.wref
        dy = dy.contiguous()
        if ctx.gathered and _use_fused(pctx, dy, x.shape[0] // pctx.tp_size):
            from ..ops import fused_tp
            dx = fused_tp.matmul_reduce_scatter(dy, w, pctx, transpose_b=True)
            X = x
        elif ctx.gathered:
            dx = _rs(ops.mm_nt(dy, w), pctx)
            X = x
        else:
            dX = ops.mm_nt(dy, w)
            dx = _rs(dX, pctx) if mode == "ag" else (_ar(dX, pctx) if mode == "f" else dX)
            X = _ag(x, pctx) if mode == "ag" else x
        grads = wref.accumulate(ops.mm_tn_acc, X, dy)
        return (dx, None, None, None, None, *grads)


def column_linear(x, wref: WeightRef, pctx: ParallelContext, mode: str, dtype: torch.dtype):
    return _ColumnLinear.apply(x, wref, pctx, mode, dtype, *wref.params)


# ------------------------------------------------- gate|up linear + SwiGLU
class _GateUpSwiGLU(torch.autograd.Function):
    """``a = silu(X W_gate) * (X W_up)`` in one GEMM whose epilogue applies the
    SwiGLU (``X = x``, or ``AG(x)`` in mode ``"ag"``): the pre-activation is
    written only when a backward will read it, and no separate element-wise
    pass reads it back. Backward: SwiGLU backward, then the column-parallel
    backward of the gate|up projection (``nano_megatron/model.py:151-152``)."""

    @staticmethod
    def forward(ctx, x, wref, pctx, mode, dtype, *params):
        x = x if x.dtype == dtype else x.to(dtype)
        w = wref.for_compute(dtype)
        keep = not _discarded_forward[0]
        ctx.gathered = mode == "ag" and _use_fused(pctx, x, x.shape[0])
        if ctx.gathered:
            from ..ops import fused_tp
            X, a, gu = fused_tp.all_gather_matmul_swiglu(x, w, pctx, save_gu=keep, save_gathered=keep)
            if X is None:
                X = _placeholder((a.shape[0], x.shape[1]), x)
            saved_x = X
        else:
            X = _ag(x, pctx) if mode == "ag" else x
            a, gu = ops.cuda_ops().mm_swiglu(X, w, save_gu=keep)
            saved_x = x
        if gu is None:
            gu = _placeholder((a.shape[0], 2 * a.shape[1]), a)
        ctx.save_for_backward(saved_x, w, gu)
        ctx.wref, ctx.pctx, ctx.mode = wref, pctx, mode
        return a

    @staticmethod
    def backward(ctx, da):
        x, w, gu = ctx.saved_tensors
        pctx, mode, wref = ctx.pctx, ctx.mode, ctx.wref
        dgu = ops.swiglu_bwd(da.contiguous(), gu)
        if ctx.gathered and _use_fused(pctx, dgu, x.shape[0] // pctx.tp_size):
            from ..ops import fused_tp
            dx = fused_tp.matmul_reduce_scatter(dgu, w, pctx, transpose_b=True)
            X = x  # the gathered input the forward kernel saved
        elif ctx.gathered:
            dx = _rs(ops.mm_nt(dgu, w), pctx)
            X = x
        else:
            dX = ops.mm_nt(dgu, w)
            dx = _rs(dX, pctx) if mode == "ag" else (_ar(dX, pctx) if mode == "f" else dX)
            X = _ag(x, pctx) if mode == "ag" else x
        grads = wref.accumulate(ops.mm_tn_acc, X, dgu)
        return (dx, None, None, None, None, *grads)


def gate_up_swiglu_supported(x: torch.Tensor, ffn_local: int, pctx: ParallelContext, mode: str) -> bool:
    """The one-GEMM SwiGLU path (bf16 compute, CUDA, 8-aligned width); with
    sequence parallelism over more than one GPU it is the fused all-gather
    kernel's SwiGLU mode."""
    return x.is_cuda and ffn_local % 8 == 0


def gate_up_swiglu(x, wref: WeightRef, pctx: ParallelContext, mode: str, dtype: torch.dtype):
    return _GateUpSwiGLU.apply(x, wref, pctx, mode, dtype, *wref.params)


# --------------------------------------------------------------- row linear
class _RowLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, wref, pctx, mode, dtype, *params):
        x = x if x.dtype == dtype else x.to(dtype)
        w = wref.for_compute(dtype)
        if mode == "rs" and _use_fused(pctx, x, x.shape[0] // pctx.tp_size):
            from ..ops import fused_tp
            y = fused_tp.matmul_reduce_scatter(x, w, pctx, transpose_b=False)
        else:
            y = ops.mm_nn(x, w)
            if mode == "rs":
                y = _rs(y, pctx)
            elif mode == "g":
                y = _ar(y, pctx)
        ctx.save_for_backward(x, w)
        ctx.wref, ctx.pctx, ctx.mode = wref, pctx, mode
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        pctx, mode, wref = ctx.pctx, ctx.mode, ctx.wref
        dy = dy.contiguous()
        if mode == "rs" and _use_fused(pctx, dy, dy.shape[0]):
            from ..ops import fused_tp
            dY, dx = fused_tp.all_gather_matmul(dy, w, pctx, transpose_b=True, return_gathered=True)
        else:
            dY = _ag(dy, pctx) if mode == "rs" else dy
            dx = ops.mm_nt(dY, w)
        grads = wref.accumulate(ops.mm_tn_acc, x, dY)
        return (dx, None, None, None, None, *grads)


def row_linear(x, wref: WeightRef, pctx: ParallelContext, mode: str, dtype: torch.dtype):
    return _RowLinear.apply(x, wref, pctx, mode, dtype, *wref.params)


# ------------------------------------------------------------------ RMSNorm
class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        y, rstd = ops.rmsnorm(x, weight.detach(), eps)
        ctx.save_for_backward(x, weight, rstd)
        ctx.main_grad = getattr(weight, "main_grad", None)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight, rstd = ctx.saved_tensors
        main_grad = ctx.main_grad
        dx, dw = ops.rmsnorm_bwd(dy.contiguous(), x, weight.detach(), rstd, main_grad)
        if main_grad is not None:
            _grad_written(main_grad)
        return dx, (None if main_grad is not None else dw.to(weight.dtype)), None


def rms_norm(x, weight, eps):
    return _RMSNorm.apply(x, weight, eps)


class _AddRMSNorm(torch.autograd.Function):
    """The residual add after a sublayer and the norm that follows it:
    ``s = x + a`` and ``h = rmsnorm(s) * w`` in one pass
    (``nano_megatron/model.py:165-166``). Backward: the norm's input gradient
    plus the residual-stream gradient of ``s`` in one pass; that sum is the
    gradient of both ``x`` and ``a``."""

    @staticmethod
    def forward(ctx, x, a, weight, eps):
        s, h, rstd = ops.add_rmsnorm(x, a, weight.detach(), eps)
        ctx.save_for_backward(s, weight, rstd)
        ctx.main_grad = getattr(weight, "main_grad", None)
        return s, h

    @staticmethod
    def backward(ctx, ds, dh):
        s, weight, rstd = ctx.saved_tensors
        main_grad = ctx.main_grad
        if dh is None:  # h unused: the add alone
            return ds, ds, None, None
        dx, dw = ops.rmsnorm_bwd(dh.contiguous(), s, weight.detach(), rstd, main_grad,
                                 None if ds is None else ds.contiguous())
        if main_grad is not None:
            _grad_written(main_grad)
        return dx, dx, (None if main_grad is not None else dw.to(weight.dtype)), None


def add_rms_norm(x, a, weight, eps):
    """``(x + a, rmsnorm(x + a) * weight)`` for 2-D ``x``, ``a`` of one shape."""
    return _AddRMSNorm.apply(x, a, weight, eps)


# ---------------------------------------------------------------- attention
class _Attention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, batch, heads, head_dim, cos, sin):
        if qkv.is_cuda:  # the QKV GEMM output is private to this op: rotate it in place
            o, saved = ops.cuda_ops().attention(qkv, batch, heads, head_dim, cos, sin, inplace=True)
        else:
            o, saved = ops.attention(qkv.contiguous(), batch, heads, head_dim, cos, sin)
        ctx.save_for_backward(*saved)
        ctx.meta = (batch, heads, head_dim)
        ctx.rope = (cos, sin)
        return o

    @staticmethod
    def backward(ctx, do):
        batch, heads, head_dim = ctx.meta
        cos, sin = ctx.rope
        dqkv = ops.attention_bwd(do.contiguous(), ctx.saved_tensors, batch, heads, head_dim, cos, sin)
        return dqkv, None, None, None, None, None


def causal_attention(qkv, batch, heads, head_dim, cos, sin):
    """RoPE + causal MHA over a fused ``[S*b, 3*h*d]`` QKV buffer -> ``[S*b, h*d]``."""
    return _Attention.apply(qkv, batch, heads, head_dim, cos, sin)


# ------------------------------------------------------------------- SwiGLU
class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        ctx.save_for_backward(gu)
        return ops.swiglu(gu.contiguous())

    @staticmethod
    def backward(ctx, da):
        (gu,) = ctx.saved_tensors
        return ops.swiglu_bwd(da.contiguous(), gu)


def swiglu(gu):
    return _SwiGLU.apply(gu)


# ---------------------------------------------------------------- embedding
class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, wref, pctx, mode, vocab_start, vocab_end, out_dtype, *params):
        if ids.is_cuda:
            vocab = (vocab_end - vocab_start) * pctx.tp_size
            y = ops.cuda_ops().embedding(ids, wref.data.detach(), vocab_start, vocab_end, out_dtype, vocab)
        else:
            y = ops.embedding(ids, wref.data.detach(), vocab_start, vocab_end)
        if pctx.tp_size > 1:
            y = _rs(y, pctx) if mode == "rs" else _ar(y, pctx)
        ctx.save_for_backward(ids)
        ctx.wref, ctx.pctx, ctx.mode, ctx.vrange = wref, pctx, mode, (vocab_start, vocab_end)
        return y

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        pctx, wref = ctx.pctx, ctx.wref
        dy = dy.contiguous()
        if pctx.tp_size > 1 and ctx.mode == "rs":
            dy = _ag(dy, pctx)
        grads = wref.accumulate(lambda d, i, out: ops.embedding_bwd(d, i, out, *ctx.vrange), dy, ids)
        return (None, None, None, None, None, None, None, *grads)


def vocab_embedding(ids, wref, pctx, mode, vocab_start, vocab_end, out_dtype):
    return _Embedding.apply(ids, wref, pctx, mode, vocab_start, vocab_end, out_dtype, *wref.params)


# -------------------------------------------------- cross-entropy statistics
def merge_ce_stats(mx, se, tl, pctx: ParallelContext):
    """Combine per-shard ``(max, sumexp, target logit)`` into global ``(M, S, target)``.

    One all-gather of a ``[3, T]`` block replaces the reference's three
    all-reduces (``cross_entropy.py:23,38,43``):
    ``M = max_r m_r``, ``S = sum_r s_r * exp(m_r - M)``, ``target = sum_r t_r``.
    """
    if pctx.tp_size == 1:
        return mx, se, tl
    stats = torch.stack([mx, se, tl]).contiguous()
    gathered = torch.empty((pctx.tp_size * 3, stats.shape[1]), dtype=stats.dtype, device=stats.device)
    dist.all_gather_into_tensor(gathered, stats, group=pctx.tp_group)
    gathered = gathered.view(pctx.tp_size, 3, -1)
    gm = gathered[:, 0].max(dim=0).values
    gs = (gathered[:, 1] * (gathered[:, 0] - gm).exp()).sum(0)
    gt = gathered[:, 2].sum(0)
    return gm, gs, gt


class _LMHeadCE(torch.autograd.Function):
    """Vocab-parallel LM head + cross entropy; returns the mean token loss.

    On CUDA in bf16 the forward is the fused kernel pair of
    :func:`nano_megatron_b200.ops.fused_tp.lm_head_cross_entropy` (all-gather,
    GEMM with the per-token statistics in its epilogue, one cross-rank merge);
    the backward turns the saved bf16 logits into ``(softmax - onehot) * g/n``
    in place and runs dgrad (fused with the reduce-scatter under sequence
    parallelism) and wgrad on them.
    """

    @staticmethod
    def forward(ctx, x, labels, wref, pctx, mode, dtype, vocab_start, vocab_end, *params):
        x = x if x.dtype == dtype else x.to(dtype)
        w = wref.for_compute(dtype)  # [V/t, H]
        ctx.fused = _use_fused_ce(pctx, x, w, mode)
        if ctx.fused:
            from ..ops import fused_tp
            loss_tok, logits, gm, gs, X = fused_tp.lm_head_cross_entropy(
                x, w, labels, vocab_start, vocab_end, pctx, gather=mode == "ag")
            ctx.save_for_backward(X, labels, w, logits, gm, gs)
        else:
            X = _ag(x, pctx) if mode == "ag" else x
            if X.is_cuda:
                loss_tok, state = ops.cuda_ops().lm_head_ce_fwd(X, w, labels, vocab_start, vocab_end, pctx)
            else:
                logits = ops.mm_nt(X, w)
                mx, se, tl, _ = ops.ce_local_stats(logits, labels, vocab_start, vocab_end)
                gm, gs, gt = merge_ce_stats(mx, se, tl, pctx)
                loss_tok = gs.log() + gm - gt
                state = (logits, gm, gs)
            ctx.save_for_backward(x, labels, w, *state)
        ctx.wref, ctx.pctx, ctx.mode, ctx.vrange, ctx.dtype = wref, pctx, mode, (vocab_start, vocab_end), dtype
        return loss_tok.mean()

    @staticmethod
    def backward(ctx, g):
        x, labels, w, *state = ctx.saved_tensors
        pctx, mode, wref = ctx.pctx, ctx.mode, ctx.wref
        n = labels.numel()
        if ctx.fused:
            X = x  # the gathered input saved by the forward kernel
            dlogits = ops.cuda_ops().lm_head_ce_grad(X, w, labels, ctx.vrange[0], state, g / n, inplace=True)
            rows_local = X.shape[0] // pctx.tp_size
            if mode == "ag" and _use_fused(pctx, dlogits, rows_local):
                from ..ops import fused_tp
                dx = fused_tp.matmul_reduce_scatter(dlogits, w, pctx, transpose_b=False)
            else:
                dX = ops.mm_nn(dlogits, w)
                dx = _rs(dX, pctx) if mode == "ag" else (_ar(dX, pctx) if mode == "f" else dX)
            grads = wref.accumulate(ops.mm_tn_acc, dlogits, X)
            return (dx, None, None, None, None, None, None, None, *grads)
        X = _ag(x, pctx) if mode == "ag" else x
        if X.is_cuda:
            dlogits = ops.cuda_ops().lm_head_ce_grad(X, w, labels, ctx.vrange[0], state, g / n)
        else:
            logits, gm, gs = state
            scale = (g / n).expand(n).float()
            dlogits = ops.ce_grad(logits, labels, ctx.vrange[0], gm, gs, scale, ctx.dtype)
        dX = ops.mm_nn(dlogits, w)
        if mode == "ag":
            dx = _rs(dX, pctx)
        elif mode == "f":
            dx = _ar(dX, pctx)
        else:
            dx = dX
        grads = wref.accumulate(ops.mm_tn_acc, dlogits, X)
        return (dx, None, None, None, None, None, None, None, *grads)


def lm_head_cross_entropy(x, labels, wref, pctx, mode, dtype, vocab_start, vocab_end):
    return _LMHeadCE.apply(x, labels, wref, pctx, mode, dtype, vocab_start, vocab_end, *wref.params)


class _LMHeadLogits(torch.autograd.Function):
    """``logits = AG(x) @ W^T`` for a vocab-sharded ``W [V/tp, H]`` (no loss)."""

    @staticmethod
    def forward(ctx, x, wref, pctx, mode, dtype, *params):
        x = x if x.dtype == dtype else x.to(dtype)
        w = wref.for_compute(dtype)
        X = _ag(x, pctx) if mode == "ag" else x
        ctx.save_for_backward(x, w)
        ctx.wref, ctx.pctx, ctx.mode = wref, pctx, mode
        return ops.mm_nt(X, w)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        pctx, mode, wref = ctx.pctx, ctx.mode, ctx.wref
        dy = dy.contiguous()
        X = _ag(x, pctx) if mode == "ag" else x
        dX = ops.mm_nn(dy, w)
        dx = _rs(dX, pctx) if mode == "ag" else (_ar(dX, pctx) if mode == "f" else dX)
        grads = wref.accumulate(ops.mm_tn_acc, dy, X)
        return (dx, None, None, None, None, *grads)


def lm_head_logits(x, wref, pctx, mode, dtype):
    return _LMHeadLogits.apply(x, wref, pctx, mode, dtype, *wref.params)
