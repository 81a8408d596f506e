"""CUDA implementations of the op layer, on the in-tree sm_100a extension.

Importing this module loads ``nano_megatron_b200/_C*.so`` and raises if it is
missing or was not built for this GPU: there is no silent fallback to
PyTorch kernels on the CUDA path.

GEMMs run the tcgen05 kernel of ``csrc/gemm.cu`` in bf16. The reference's
``--dtype float32`` mode runs the exact-fp32 SIMT kernels of ``csrc/fp32.cu``
(strided GEMM, materialized causal softmax attention): correct to fp32
tolerances, not fast; bf16 is the performance path.
"""

from __future__ import annotations

import torch

try:
    from .. import _C  # noqa: F401
except ImportError as exc:  # pragma: no cover - exercised only without a build
    raise ImportError(
        "nano_megatron_b200._C is not built; run `python setup.py build_ext --inplace` "
        "(or __graft_entry__.build()) before using CUDA tensors") from exc

from .. import _C as C  # noqa: E402

_status: dict[int, torch.Tensor] = {}

# Number of our kernels launched so far (benchmarks read the difference
# around a timed region; each wrapper adds the kernels it launches).
LAUNCHES = [0]


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n


_partial_cache: dict[tuple, torch.Tensor] = {}

ERROR_MESSAGES = {1: "an mbarrier wait timed out inside a kernel",
                  2: "a cross-GPU flag wait timed out",
                  3: "a token id is outside the vocabulary",
                  4: "a kernel was launched with an unsupported shape"}


def status_word(device: torch.device) -> torch.Tensor:
    """The device's int32 error word that bounded waits and bounds checks write."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


class CollectiveTimeout(RuntimeError):
    """A kernel gave up waiting for another GPU (a peer stopped, or never started)."""


def check_status(device: torch.device | None = None) -> None:
    """Raise if any kernel on ``device`` reported an error since the last check (syncs).

    Code 2 (a cross-GPU flag wait ran out) raises :class:`CollectiveTimeout`.
    """
    device = device or torch.device("cuda", torch.cuda.current_device())
    word = status_word(device)
    code = int(word[0].item())
    if code:
        word.zero_()
        _raise_for(code)


def _raise_for(code: int) -> None:
    cls = CollectiveTimeout if code == 2 else RuntimeError
    raise cls(f"CUDA kernel error {code}: {ERROR_MESSAGES.get(code, 'unknown')}")


class StatusPoller:
    """Checks the status word without stalling the host on the device.

    ``poll()`` looks at the last snapshot whose copy has completed (an event
    query, no synchronization), raises if it holds an error, and enqueues a
    fresh snapshot (a 16-byte device->pinned-host copy on the current stream)
    when none is in flight. Errors are therefore reported one or two steps
    after the kernel that set them; ``final()`` synchronizes and checks
    everything up to now (call it before exiting).
    """

    def __init__(self, device: torch.device):
        self.device = device
        self.host = torch.zeros(4, dtype=torch.int32, pin_memory=True)
        self.event: torch.cuda.Event | None = None

    def poll(self) -> None:
        if self.event is not None:
            if not self.event.query():
                return
            self.event = None
            code = int(self.host[0])
            if code:
                status_word(self.device).zero_()
                _raise_for(code)
        self.host.copy_(status_word(self.device), non_blocking=True)
        self.event = torch.cuda.Event()
        self.event.record()

    def final(self) -> None:
        torch.cuda.synchronize(self.device)
        self.event = None
        check_status(self.device)


def _dtype_ok(t: torch.Tensor) -> None:
    if t.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"unsupported dtype {t.dtype}")


# --------------------------------------------------------------------- GEMM
def _gemm(a, b, c, a_mn, b_mn, out_mode):
    C.gemm(a, b, c, a_mn, b_mn, out_mode, status_word(a.device))
    _count()


def _f32_gemm(a, b, a_t, b_t, out=None, beta=0.0):
    """Exact fp32 ``op(a) @ op(b)`` (SIMT FMA kernel, no TF32), optionally ``+= out``."""
    m = a.shape[1] if a_t else a.shape[0]
    n = b.shape[0] if b_t else b.shape[1]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=a.device)
    C.gemm_f32(a, b, out, a_t, b_t, beta)
    _count()
    return out


def mm_nn(a, b):
    """``a[M,K] @ b[K,N]``."""
    if a.dtype == torch.float32:
        return _f32_gemm(a, b, False, False)
    out = torch.empty((a.shape[0], b.shape[1]), dtype=a.dtype, device=a.device)
    _gemm(a, b, out, False, True, 0)
    return out


def mm_nt(a, b):
    """``a[M,K] @ b[N,K]^T``."""
    if a.dtype == torch.float32:
        return _f32_gemm(a, b, False, True)
    out = torch.empty((a.shape[0], b.shape[0]), dtype=a.dtype, device=a.device)
    _gemm(a, b, out, False, False, 0)
    return out


def mm_swiglu(x, w_gu, save_gu: bool):
    """``silu(x @ w_gate) * (x @ w_up)`` for the fused ``w_gu = [w_gate | w_up]``
    ``[K, 2F]`` in one GEMM (SwiGLU epilogue); also the pre-activation
    ``gu [M, 2F]`` when ``save_gu`` (the backward needs it), else None."""
    m, f = x.shape[0], w_gu.shape[1] // 2
    a = torch.empty((m, f), dtype=x.dtype, device=x.device)
    gu = torch.empty((m, 2 * f), dtype=x.dtype, device=x.device) if save_gu else None
    C.gemm_swiglu(x, w_gu, a, gu, status_word(x.device))
    _count()
    return a, gu


def mm_tn_acc(a, b, out):
    """``out[K,N] += a[M,K]^T @ b[M,N]`` (fp32 ``out``)."""
    if a.dtype == torch.float32:
        _f32_gemm(a, b, True, False, out=out, beta=1.0)
        return
    if out.stride(-1) != 1:
        raise ValueError("accumulator must have unit inner stride")
    _gemm(a, b, out, True, True, 2)


# ------------------------------------------------------------------ RMSNorm
def rmsnorm(x, weight, eps):
    _dtype_ok(x)
    x = x.contiguous()
    y = torch.empty_like(x)
    rstd = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    C.rmsnorm_fwd(x, weight.contiguous().float(), y, rstd, float(eps))
    _count()
    return y, rstd


def _partial(device, rows, cols):
    key = (device.index, rows, cols)
    buf = _partial_cache.get(key)
    if buf is None:
        buf = torch.empty((rows, cols), dtype=torch.float32, device=device)
        _partial_cache[key] = buf
    return buf


def add_rmsnorm(x, a, weight, eps):
    """``s = x + a`` and ``(rmsnorm(s) * weight, rstd)`` in one pass: ``(s, y, rstd)``."""
    _dtype_ok(x)
    x, a = x.contiguous(), a.contiguous()
    s, y = torch.empty_like(x), torch.empty_like(x)
    rstd = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    C.add_rmsnorm_fwd(x, a, s, weight.contiguous().float(), y, rstd, float(eps))
    _count()
    return s, y, rstd


def rmsnorm_bwd(dy, x, weight, rstd, wgrad_out, dres=None):
    dx = torch.empty_like(x)
    nblk = C.rmsnorm_bwd_blocks(x.shape[0])
    part = _partial(x.device, nblk, x.shape[1])
    C.rmsnorm_bwd(dy.contiguous(), x, weight.contiguous().float(), rstd, dx, part,
                  None if dres is None else dres.contiguous())
    _count(2)
    if wgrad_out is not None:
        C.reduce_rows_add(part, nblk, wgrad_out)
        return dx, None
    dw = torch.zeros(x.shape[1], dtype=torch.float32, device=x.device)
    C.reduce_rows_add(part, nblk, dw)
    return dx, dw


# ---------------------------------------------------------------- attention
def _attention_f32(qkv, batch, heads, head_dim, cos, sin):
    """fp32 causal attention, materialized per (batch, head) with the fp32 kernels."""
    qkv = qkv.clone(memory_format=torch.contiguous_format)
    C.rope_inplace(qkv, cos, sin, batch, heads, head_dim, 1.0)
    s = qkv.shape[0] // batch
    t = qkv.view(s, batch, 3, heads, head_dim)
    o = torch.empty((qkv.shape[0], heads * head_dim), dtype=qkv.dtype, device=qkv.device)
    ov = o.view(s, batch, heads, head_dim)
    probs = torch.empty((batch, heads, s, s), dtype=torch.float32, device=qkv.device)
    scores = torch.empty((s, s), dtype=torch.float32, device=qkv.device)
    scale = head_dim ** -0.5
    for bi in range(batch):
        for h in range(heads):
            q, k, v = t[:, bi, 0, h], t[:, bi, 1, h], t[:, bi, 2, h]
            _f32_gemm(q, k, False, True, out=scores)
            C.causal_softmax_f32(scores, probs[bi, h], scale)
            C.gemm_f32(probs[bi, h], v, ov[:, bi, h], False, False, 0.0)
            _count(2)
    _count()
    return o, (qkv, probs)


def _attention_bwd_f32(do, saved, batch, heads, head_dim, cos, sin):
    qkv, probs = saved
    s = qkv.shape[0] // batch
    t = qkv.view(s, batch, 3, heads, head_dim)
    dqkv = torch.empty_like(qkv)
    dt = dqkv.view(s, batch, 3, heads, head_dim)
    dov = do.view(s, batch, heads, head_dim)
    dp = torch.empty((s, s), dtype=torch.float32, device=qkv.device)
    ds = torch.empty_like(dp)
    scale = head_dim ** -0.5
    for bi in range(batch):
        for h in range(heads):
            q, k, v = t[:, bi, 0, h], t[:, bi, 1, h], t[:, bi, 2, h]
            p, g = probs[bi, h], dov[:, bi, h]
            C.gemm_f32(p, g, dt[:, bi, 2, h], True, False, 0.0)      # dV = P^T dO
            C.gemm_f32(g, v, dp, False, True, 0.0)                   # dP = dO V^T
            C.softmax_bwd_f32(p, dp, ds, scale)                      # dS (scaled)
            C.gemm_f32(ds, k, dt[:, bi, 0, h], False, False, 0.0)    # dQ = dS K
            C.gemm_f32(ds, q, dt[:, bi, 1, h], True, False, 0.0)     # dK = dS^T Q
            _count(5)
    C.rope_inplace(dqkv, cos, sin, batch, heads, head_dim, -1.0)
    _count()
    return dqkv


def attention(qkv, batch, heads, head_dim, cos, sin, inplace=False):
    """RoPE + causal flash attention. With ``inplace`` the rotation is applied
    to ``qkv`` itself (the model passes its private QKV GEMM output). fp32
    inputs take the exact-fp32 materialized path; so do bf16 inputs the flash
    kernels do not cover (head size other than 128, or a sequence length that
    is not a multiple of 64), upcast and with the output cast back: any head
    size that is a multiple of 16 and any length run, at O(S^2) memory per
    (batch, head) pair."""
    if qkv.dtype == torch.float32:
        return _attention_f32(qkv, batch, heads, head_dim, cos, sin)
    if head_dim != 128 or (qkv.shape[0] // batch) % 64 != 0:
        o, saved = _attention_f32(qkv.float(), batch, heads, head_dim, cos, sin)
        return o.to(qkv.dtype), saved
    qkv = qkv.contiguous() if inplace else qkv.clone(memory_format=torch.contiguous_format)
    C.rope_inplace(qkv, cos, sin, batch, heads, head_dim, 1.0)
    if (qkv.shape[0] // batch) % 128 == 0:
        o, lse = C.flash_attn_fwd_tc(qkv, batch, heads, head_dim, status_word(qkv.device))
    else:  # sequence lengths that are not a multiple of 128: mma.sync kernel
        o, lse = C.flash_attn_fwd(qkv, batch, heads, head_dim)
    _count(2)
    return o, (qkv, o, lse)


def attention_bwd(do, saved, batch, heads, head_dim, cos, sin):
    if len(saved) == 2:  # the materialized path (fp32, or bf16 with a head size other than 128)
        dqkv = _attention_bwd_f32(do.float().contiguous(), saved, batch, heads, head_dim, cos, sin)
        return dqkv if do.dtype == torch.float32 else dqkv.to(do.dtype)
    qkv, o, lse = saved
    if (qkv.shape[0] // batch) % 128 == 0:
        # the inverse RoPE is applied to dQ and dK as the kernels store them
        dqkv = C.flash_attn_bwd_tc(do.contiguous(), qkv, o, lse, batch, heads, head_dim, status_word(qkv.device),
                                   cos.contiguous(), sin.contiguous())
        _count(4)  # D = rowsum(dO * O), lse scaling, dK/dV kernel, dQ kernel
    else:
        dqkv = C.flash_attn_bwd(do.contiguous(), qkv, o, lse, batch, heads, head_dim)
        C.rope_inplace(dqkv, cos, sin, batch, heads, head_dim, -1.0)
        _count(4)
    return dqkv


# ------------------------------------------------------------------- SwiGLU
def swiglu(gu):
    a = torch.empty((gu.shape[0], gu.shape[1] // 2), dtype=gu.dtype, device=gu.device)
    C.swiglu_fwd(gu.contiguous(), a)
    _count()
    return a


def swiglu_bwd(da, gu):
    dgu = torch.empty_like(gu)
    C.swiglu_bwd(da.contiguous(), gu.contiguous(), dgu)
    _count()
    return dgu


# ---------------------------------------------------------------- embedding
def embedding(ids, weight, vocab_start, vocab_end, out_dtype=None, vocab_size=None):
    ids = ids.contiguous()
    out = torch.empty((ids.numel(), weight.shape[1]), dtype=out_dtype or weight.dtype, device=weight.device)
    vocab = vocab_size if vocab_size is not None else 1 << 62
    C.embedding_fwd(ids, weight.contiguous(), out, vocab_start, vocab_end, vocab, status_word(weight.device))
    _count()
    return out


def embedding_bwd(dy, ids, wgrad_out, vocab_start, vocab_end):
    C.embedding_bwd(dy.contiguous(), ids.contiguous(), wgrad_out, vocab_start, vocab_end)
    _count()


# ------------------------------------------------------------ cross entropy
def ce_local_stats(logits, target, vocab_start, vocab_end):
    n = logits.shape[0]
    mx = torch.empty(n, dtype=torch.float32, device=logits.device)
    se = torch.empty_like(mx)
    tl = torch.empty_like(mx)
    C.ce_stats(logits, target.contiguous(), mx, se, tl, vocab_start)
    _count()
    return mx, se, tl, None


# The CE-gradient kernel launches one grid row per token, and a grid has at
# most 65535 rows; longer inputs run as consecutive launches over row blocks.
_CE_GRAD_MAX_ROWS = 65535
_CE_GRAD_BLOCK_ROWS = 32768


def _ce_grad_launch(logits, target, gmax, gsum, scale1, d, vocab_start) -> None:
    rows = logits.shape[0]
    if rows <= _CE_GRAD_MAX_ROWS:
        C.ce_grad(logits, target, gmax, gsum, scale1, 1.0, d, vocab_start)
        _count()
        return
    for r0 in range(0, rows, _CE_GRAD_BLOCK_ROWS):
        r1 = min(rows, r0 + _CE_GRAD_BLOCK_ROWS)
        C.ce_grad(logits[r0:r1], target[r0:r1], gmax[r0:r1], gsum[r0:r1], scale1, 1.0, d[r0:r1], vocab_start)
        _count()


def ce_grad(logits, target, vocab_start, gmax, gsum, scale, out_dtype):
    """``scale`` may be a per-row tensor (generic path) or a device scalar."""
    d = torch.empty(logits.shape, dtype=logits.dtype, device=logits.device)
    if scale.numel() == 1:
        _ce_grad_launch(logits, target.contiguous(), gmax, gsum, scale.float().reshape(1), d, vocab_start)
        return d if d.dtype == out_dtype else d.to(out_dtype)
    _ce_grad_launch(logits, target.contiguous(), gmax, gsum, torch.ones(1, device=logits.device), d,
                    vocab_start)
    d = d * scale.unsqueeze(-1).to(d.dtype)
    return d if d.dtype == out_dtype else d.to(out_dtype)


def lm_head_ce_fwd(X, w, labels, vocab_start, vocab_end, pctx):
    """LM-head logits + per-token loss. Returns ``(loss [T], state)``."""
    from ..models.functional import merge_ce_stats
    logits = mm_nt(X, w)
    mx, se, tl, _ = ce_local_stats(logits, labels, vocab_start, vocab_end)
    gm, gs, gt = merge_ce_stats(mx, se, tl, pctx)
    loss = gs.log() + gm - gt
    return loss, (logits, gm, gs)


def lm_head_ce_grad(X, w, labels, vocab_start, state, g_over_n, inplace=False):
    """``(softmax - onehot) * g/n`` from the saved logits; ``inplace`` overwrites them."""
    logits, gm, gs = state
    d = logits if inplace else torch.empty_like(logits)
    if inplace:
        torch.autograd.graph.increment_version(logits)
    _ce_grad_launch(logits, labels.contiguous(), gm, gs, g_over_n.float().reshape(1), d, vocab_start)
    return d


# -------------------------------------------------------------- optimizer
def adamw_flat(p, g, m, v, compute, scale, *, lr, beta1, beta2, eps, weight_decay, step):
    C.adamw_flat(p, g, m, v, compute, scale.reshape(1), lr, beta1, beta2, eps, weight_decay, step)
    _count()


_norm_tables: dict[tuple, tuple] = {}
_CHUNK = 1 << 24


def weighted_sq_norm(tensors, weights):
    """``sum_i w_i * ||t_i||^2`` in fp64 (fp32 tensors, any strides of views into one buffer)."""
    device = tensors[0].device
    key = tuple((t.data_ptr(), t.numel(), w) for t, w in zip(tensors, weights))
    table = _norm_tables.get(key)
    if table is None:
        ptrs, numels, ws = [], [], []
        # Views of the flat buffer may be column slices; merge by storage span.
        for t, w in zip(tensors, weights):
            if not t.is_contiguous():
                raise ValueError("norm segments must be contiguous")
            base, n = t.data_ptr(), t.numel()
            for off in range(0, n, _CHUNK):
                ptrs.append(base + off * 4)
                numels.append(min(_CHUNK, n - off))
                ws.append(w)
        table = (torch.tensor(ptrs, dtype=torch.int64, device=device),
                 torch.tensor(numels, dtype=torch.int64, device=device),
                 torch.tensor(ws, dtype=torch.float64, device=device))
        _norm_tables[key] = table
    out = torch.zeros((), dtype=torch.float64, device=device)
    C.weighted_sq_norm(*table, out)
    _count()
    return out
