"""Plain-PyTorch implementations of every op, used on CPU.

These are the numerical oracle: the CPU/Gloo path runs them, and each CUDA
kernel's test compares against them computed in fp32. Shapes use the
framework's token-major, sequence-first layout: a ``[T, C]`` activation has
row ``t = s * batch + b``.

Semantics follow ``nano_megatron/model.py`` (RMSNorm 65-75, RoPE 78-89,
attention 113-128, SwiGLU 150-153), ``nano_megatron/tp_layers.py`` (embedding
112-132) and ``nano_megatron/cross_entropy.py`` (16-65).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


# --------------------------------------------------------------------- GEMM
def mm_nn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a[M,K] @ b[K,N]`` in the inputs' dtype."""
    return a @ b


def mm_nt(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a[M,K] @ b[N,K]^T``."""
    return a @ b.t()


def mm_tn_acc(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor) -> None:
    """``out[K,N] += a[M,K]^T @ b[M,N]`` with ``out`` fp32."""
    out.add_((a.t() @ b).to(out.dtype))


# ------------------------------------------------------------------ RMSNorm
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float):
    """Return ``(y, rstd)``; statistics in fp32, output in ``x.dtype``."""
    xf = x.float()
    rstd = xf.pow(2).mean(-1, keepdim=True).add(eps).rsqrt()
    y = (xf * rstd).to(x.dtype) * weight.to(x.dtype)
    return y, rstd.squeeze(-1)


def add_rmsnorm(x: torch.Tensor, a: torch.Tensor, weight: torch.Tensor, eps: float):
    """``s = x + a`` (in ``x.dtype``) and ``rmsnorm(s)``: returns ``(s, y, rstd)``."""
    s = x + a
    y, rstd = rmsnorm(s, weight, eps)
    return s, y, rstd


def rmsnorm_bwd(dy: torch.Tensor, x: torch.Tensor, weight: torch.Tensor,
                rstd: torch.Tensor, wgrad_out: torch.Tensor | None, dres: torch.Tensor | None = None):
    """Gradient of :func:`rmsnorm`; adds the weight gradient into ``wgrad_out``
    and, when given, the residual-stream gradient ``dres`` into ``dx``.

    Returns ``(dx, dweight)``; ``dweight`` is None when it was accumulated.
    """
    xf = x.float()
    r = rstd.unsqueeze(-1)
    xhat = xf * r
    dyf = dy.float()
    # y = cast(xhat) * w  (the cast is treated as identity for the gradient)
    dw = (dyf * xhat.to(x.dtype).float()).sum(0)
    g = dyf * weight.float()
    dx = r * (g - xhat * (g * xhat).mean(-1, keepdim=True))
    dx = dx.to(x.dtype)
    if dres is not None:
        dx = dx + dres
    if wgrad_out is not None:
        wgrad_out.add_(dw.to(wgrad_out.dtype))
        return dx, None
    return dx, dw


# --------------------------------------------------------------------- RoPE
def rope_cache(seq_len: int, head_dim: int, theta: float, device=None):
    """fp32 ``cos, sin`` of shape ``[seq_len, head_dim/2]`` (NeoX half split)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))
    freqs = torch.outer(torch.arange(seq_len, device=device).float(), inv_freq)
    return freqs.cos(), freqs.sin()


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, sign: float):
    # x [S, b, h, d]; cos/sin [S, d/2]
    x1, x2 = x.chunk(2, dim=-1)
    c = cos[: x.shape[0]].view(x.shape[0], 1, 1, -1).to(torch.float32)
    s = sin[: x.shape[0]].view(x.shape[0], 1, 1, -1).to(torch.float32) * sign
    x1f, x2f = x1.float(), x2.float()
    return torch.cat([x1f * c - x2f * s, x2f * c + x1f * s], dim=-1).to(x.dtype)


def split_qkv(qkv: torch.Tensor, batch: int, heads: int, head_dim: int):
    """Views ``q, k, v`` of shape ``[S, b, h, d]`` into a ``[S*b, 3*h*d]`` buffer."""
    s = qkv.shape[0] // batch
    t = qkv.view(s, batch, 3, heads, head_dim)
    return t[:, :, 0], t[:, :, 1], t[:, :, 2]


# ---------------------------------------------------------------- attention
def attention(qkv: torch.Tensor, batch: int, heads: int, head_dim: int,
              cos: torch.Tensor, sin: torch.Tensor):
    """Causal MHA with RoPE on q and k. ``qkv [S*b, 3*h*d]`` -> ``o [S*b, h*d]``.

    Returns ``(o, saved)`` with ``saved = (qkv_rotated,)``: what the backward needs.
    """
    q, k, v = split_qkv(qkv, batch, heads, head_dim)
    q = _rotate(q, cos, sin, 1.0)
    k = _rotate(k, cos, sin, 1.0)
    qb, kb, vb = (t.permute(1, 2, 0, 3) for t in (q, k, v))  # [b, h, S, d]
    o = F.scaled_dot_product_attention(qb, kb, vb, is_causal=True)
    o = o.permute(2, 0, 1, 3).reshape(qkv.shape[0], heads * head_dim)
    rotated = torch.stack([q, k, v], dim=2).reshape(qkv.shape)
    return o, (rotated,)


def attention_bwd(do: torch.Tensor, saved, batch: int, heads: int,
                  head_dim: int, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Gradient w.r.t. the un-rotated ``qkv`` input of :func:`attention`."""
    (qkv_rot,) = saved
    q, k, v = (t.detach().permute(1, 2, 0, 3).requires_grad_(True)
               for t in split_qkv(qkv_rot, batch, heads, head_dim))
    with torch.enable_grad():
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        g = do.view(-1, batch, heads, head_dim).permute(1, 2, 0, 3)
        dq, dk, dv = torch.autograd.grad(o, (q, k, v), g)
    dq, dk, dv = (t.permute(2, 0, 1, 3) for t in (dq, dk, dv))  # [S, b, h, d]
    dq = _rotate(dq, cos, sin, -1.0)
    dk = _rotate(dk, cos, sin, -1.0)
    return torch.stack([dq, dk, dv], dim=2).reshape(qkv_rot.shape)


# ------------------------------------------------------------------ SwiGLU
def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` where ``gu = [gate | up]`` along the last dim."""
    g, u = gu.chunk(2, dim=-1)
    return F.silu(g) * u


def swiglu_bwd(da: torch.Tensor, gu: torch.Tensor) -> torch.Tensor:
    g, u = (t.float() for t in gu.chunk(2, dim=-1))
    daf = da.float()
    sig = torch.sigmoid(g)
    silu = g * sig
    dg = daf * u * (sig * (1 + g * (1 - sig)))
    du = daf * silu
    return torch.cat([dg, du], dim=-1).to(gu.dtype)


# --------------------------------------------------------------- embedding
def embedding(ids: torch.Tensor, weight: torch.Tensor, vocab_start: int, vocab_end: int):
    """Rows of a vocab shard; ids outside ``[vocab_start, vocab_end)`` give zero rows."""
    mask = (ids < vocab_start) | (ids >= vocab_end)
    local = (ids - vocab_start).masked_fill(mask, 0)
    y = F.embedding(local, weight)
    return y.masked_fill(mask.unsqueeze(-1), 0.0)


def embedding_bwd(dy: torch.Tensor, ids: torch.Tensor, wgrad_out: torch.Tensor,
                  vocab_start: int, vocab_end: int) -> None:
    mask = (ids < vocab_start) | (ids >= vocab_end)
    local = (ids - vocab_start).masked_fill(mask, 0)
    rows = dy.float().masked_fill(mask.unsqueeze(-1), 0.0)
    wgrad_out.index_add_(0, local, rows.to(wgrad_out.dtype))


# ------------------------------------------------------ cross entropy parts
def ce_local_stats(logits: torch.Tensor, target: torch.Tensor, vocab_start: int, vocab_end: int):
    """Per-row ``(max, sum exp(l - max), target logit or 0, owns target)`` on a vocab shard."""
    lf = logits.float()
    mx = lf.max(dim=-1).values
    se = (lf - mx.unsqueeze(-1)).exp().sum(-1)
    owned = (target >= vocab_start) & (target < vocab_end)
    local = (target - vocab_start).clamp(0, logits.shape[-1] - 1)
    tl = lf.gather(-1, local.unsqueeze(-1)).squeeze(-1)
    tl = torch.where(owned, tl, torch.zeros_like(tl))
    return mx, se, tl, owned


def ce_grad(logits: torch.Tensor, target: torch.Tensor, vocab_start: int, gmax: torch.Tensor,
            gsum: torch.Tensor, scale: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
    """``(softmax - onehot) * scale`` for one vocab shard; ``scale`` is per row."""
    p = (logits.float() - gmax.unsqueeze(-1)).exp() / gsum.unsqueeze(-1)
    local = target - vocab_start
    owned = (local >= 0) & (local < logits.shape[-1])
    rows = torch.nonzero(owned, as_tuple=True)[0]
    p[rows, local[rows]] -= 1.0
    return (p * scale.unsqueeze(-1)).to(out_dtype)


# ----------------------------------------------------------------- AdamW
def adamw_(param: torch.Tensor, grad: torch.Tensor, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor,
           *, lr: float, beta1: float, beta2: float, eps: float, weight_decay: float,
           step: int, grad_scale: float = 1.0, compute_copy: torch.Tensor | None = None) -> None:
    """One decoupled-weight-decay Adam step, the update rule of ``torch.optim.AdamW``."""
    g = grad if grad_scale == 1.0 else grad * grad_scale
    param.mul_(1 - lr * weight_decay)
    exp_avg.lerp_(g, 1 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    denom = (exp_avg_sq.sqrt() / math.sqrt(bc2)).add_(eps)
    param.addcdiv_(exp_avg, denom, value=-lr / bc1)
    if compute_copy is not None:
        compute_copy.copy_(param)


def sq_norm(t: torch.Tensor) -> torch.Tensor:
    """Sum of squares in fp64."""
    return t.detach().double().pow(2).sum()
