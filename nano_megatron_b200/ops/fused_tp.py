"""Fused tensor-parallel GEMM + sequence-parallel collectives (CUDA, NVLink peers).

Each TP group owns one symmetric workspace (allocated with
``torch.distributed._symmetric_memory`` and mapped by every rank of the group;
torch is used only to exchange the peer mappings). The kernels of
``csrc/fused_tp.cu`` read and write it directly:

* ``all_gather_matmul(x, w)``: ``AG(x) @ op(w)`` — each rank pushes its
  sequence shard into every peer's gather buffer while its GEMM starts on the
  local shard; peer chunks are consumed as they arrive.
* ``matmul_reduce_scatter(x, w)``: ``RS(x @ op(w))`` — partial output tiles go
  straight to the owning rank, which adds them to its own accumulator.
* ``lm_head_cross_entropy(x, w, labels, ...)``: the vocab-parallel LM head
  and cross entropy — all-gather -> ``AG(x) @ w^T`` whose epilogue keeps the
  per-token max / sum-exp / target logit of each logit tile, then one merge
  kernel that exchanges those three scalars per token with the other ranks
  through the workspace and writes the loss.

``op(w)`` is ``w`` (``[K, N]``) or, with ``transpose_b=True``, ``w^T`` for
``w [N, K]``. A gathered tensor returned by ``all_gather_matmul(...,
return_gathered=True)`` is a view of the workspace and is valid only until the
next fused call on this TP group.

Parity: replaces the NCCL collectives of ``nano_megatron/mappings.py:43-80``
(same values: concatenation in TP-rank order, SUM reduce-scatter) and the three
per-token all-reduces of ``nano_megatron/cross_entropy.py:21-45`` (MAX of the
max, SUM of the target logit, SUM of the rescaled exp-sum), which become one
exchange of (max, sum-exp, target) triples merged with the log-sum-exp rule.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..parallel.context import ParallelContext
from . import cuda as K

ALIGN = 1 << 16
TIMEOUT_S = 60.0


def _round(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


class TPWorkspace:
    """Symmetric workspace of one TP group: flags | gather | recv | CE exchange."""

    def __init__(self, pctx: ParallelContext, device: torch.device):
        self.pctx = pctx
        self.device = device
        self.epoch = 0
        self.ce_epoch = 0
        self.buf = None
        self.handle = None
        self.gather_bytes = 0
        self.recv_bytes = 0
        self.ce_bytes = 0
        self.flag_bytes = _round(K.C.fused_tp_flag_bytes())

    def ensure(self, gather_bytes: int, recv_bytes: int, ce_bytes: int = 0) -> None:
        if gather_bytes <= self.gather_bytes and recv_bytes <= self.recv_bytes and ce_bytes <= self.ce_bytes:
            return
        import torch.distributed._symmetric_memory as symm
        gather_bytes = max(_round(gather_bytes), self.gather_bytes)
        recv_bytes = max(_round(recv_bytes), self.recv_bytes)
        ce_bytes = max(_round(ce_bytes), self.ce_bytes)
        if self.buf is not None:
            # Every rank's kernels on the old buffer must be finished before it
            # goes. They all ran on this stream; a device-wide synchronize would
            # also wait for other streams' work (e.g. an NCCL kernel waiting for
            # a peer that is itself here), so only this stream is drained.
            torch.cuda.current_stream(self.device).synchronize()
            dist.barrier(group=self.pctx.tp_group)
        total = self.flag_bytes + gather_bytes + recv_bytes + ce_bytes
        buf = symm.empty(total, dtype=torch.uint8, device=self.device)
        buf.zero_()
        handle = symm.rendezvous(buf, self.pctx.tp_group)
        torch.cuda.current_stream(self.device).synchronize()
        dist.barrier(group=self.pctx.tp_group)
        self.buf, self.handle = buf, handle
        self.ptrs = [int(p) for p in handle.buffer_ptrs]
        self.gather_bytes, self.recv_bytes, self.ce_bytes = gather_bytes, recv_bytes, ce_bytes
        self.flags_off = 0
        self.gather_off = self.flag_bytes
        self.recv_off = self.flag_bytes + gather_bytes
        self.ce_off = self.recv_off + recv_bytes

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def next_ce_epoch(self) -> int:
        """Merge calls alternate between two data slots by the parity of this counter."""
        self.ce_epoch += 1
        return self.ce_epoch

    def gathered(self, rows: int, cols: int, dtype=torch.bfloat16) -> torch.Tensor:
        n = rows * cols * torch.empty((), dtype=dtype).element_size()
        return self.buf[self.gather_off: self.gather_off + n].view(dtype).view(rows, cols)


def workspace(pctx: ParallelContext, device: torch.device) -> TPWorkspace:
    ws = pctx.resources.get("tp_workspace")
    if ws is None:
        ws = TPWorkspace(pctx, device)
        pctx.resources["tp_workspace"] = ws
    return ws


def supported(rows_local: int, pctx: ParallelContext) -> bool:
    """Shapes the fused kernels take: 128-row multiples per rank, up to 8 ranks."""
    return pctx.tp_size <= 8 and rows_local % 128 == 0


def all_gather_matmul(x_local, w, pctx: ParallelContext, transpose_b: bool = False,
                      return_gathered: bool = False, save_gathered: bool = False):
    """``AG(x_local) @ op(w)``; with ``return_gathered`` also the gathered input.

    ``return_gathered`` gives a view of the workspace (valid until the next
    fused call); ``save_gathered`` gives a private copy that the kernel's comm
    warps write while the GEMM runs (for a later weight gradient).
    """
    x_local = x_local.contiguous()
    m_chunk, k = x_local.shape
    rows = m_chunk * pctx.tp_size
    n = w.shape[0] if transpose_b else w.shape[1]
    ws = workspace(pctx, x_local.device)
    ws.ensure(rows * k * 2, 0)
    out = torch.empty((rows, n), dtype=x_local.dtype, device=x_local.device)
    saved = torch.empty((rows, k), dtype=x_local.dtype, device=x_local.device) if save_gathered else None
    K.C.fused_tp_gemm(0, x_local, w, not transpose_b, out, ws.ptrs, pctx.tp_rank, rows, ws.gather_off,
                      ws.recv_off, ws.flags_off, ws.next_epoch(), return_gathered,
                      K.status_word(x_local.device), TIMEOUT_S, save_out=saved)
    K._count()
    if return_gathered:
        return ws.gathered(rows, k), out
    if save_gathered:
        return saved, out
    return out


def all_gather_matmul_swiglu(x_local, w_gu, pctx: ParallelContext, save_gu: bool = True,
                             save_gathered: bool = True):
    """``silu(AG(x) @ w_gate) * (AG(x) @ w_up)`` for ``w_gu = [w_gate | w_up]``
    ``[K, 2F]`` in one kernel (all-gather, GEMM, SwiGLU epilogue). Returns
    ``(X, a, gu)``: the private gathered input (None unless ``save_gathered``),
    the activation ``[M, F]`` and the pre-activation ``[M, 2F]`` (None unless
    ``save_gu``)."""
    x_local = x_local.contiguous()
    m_chunk, k = x_local.shape
    rows = m_chunk * pctx.tp_size
    f = w_gu.shape[1] // 2
    ws = workspace(pctx, x_local.device)
    ws.ensure(rows * k * 2, 0)
    a = torch.empty((rows, f), dtype=x_local.dtype, device=x_local.device)
    gu = torch.empty((rows, 2 * f), dtype=x_local.dtype, device=x_local.device) if save_gu else None
    saved = torch.empty((rows, k), dtype=x_local.dtype, device=x_local.device) if save_gathered else None
    K.C.fused_tp_gemm(3, x_local, w_gu, True, a, ws.ptrs, pctx.tp_rank, rows, ws.gather_off, ws.recv_off,
                      ws.flags_off, ws.next_epoch(), False, K.status_word(x_local.device), TIMEOUT_S,
                      save_out=saved, gu=gu)
    K._count()
    return saved, a, gu


def matmul_reduce_scatter(x, w, pctx: ParallelContext, transpose_b: bool = False):
    """``RS(x @ op(w))`` over the sequence (row) dim: returns this rank's rows."""
    x = x.contiguous()
    rows, k = x.shape
    n = w.shape[0] if transpose_b else w.shape[1]
    ws = workspace(pctx, x.device)
    ws.ensure(0, rows * n * 2)
    out = torch.empty((rows // pctx.tp_size, n), dtype=x.dtype, device=x.device)
    K.C.fused_tp_gemm(1, x, w, not transpose_b, out, ws.ptrs, pctx.tp_rank, rows, ws.gather_off,
                      ws.recv_off, ws.flags_off, ws.next_epoch(), False, K.status_word(x.device), TIMEOUT_S)
    K._count()
    return out


def ce_supported(rows_local: int, vocab_local: int) -> bool:
    return rows_local % 128 == 0 and vocab_local % 8 == 0


def lm_head_cross_entropy(x, w, labels, vocab_start: int, vocab_end: int, pctx: ParallelContext,
                          gather: bool):
    """Vocab-parallel LM head + cross entropy, fused (bf16, CUDA).

    ``x``: this rank's sequence shard ``[T/t, H]`` (``gather=True``, the kernel
    all-gathers it) or the full ``[T, H]``; ``w``: ``[V/t, H]``; ``labels``:
    ``[T]`` int64 in the row order of the gathered input. Returns ``(loss [T]
    fp32, logits [T, V/t] bf16, gmax [T], gsum [T], X)`` where ``X`` is the
    gathered input (a private copy) for the weight gradient.
    """
    x = x.contiguous()
    tp = pctx.tp_size if gather else 1
    rows = x.shape[0] * tp
    hidden = x.shape[1]
    vocab_local = w.shape[0]
    dev = x.device
    num_n = (vocab_local + 255) // 256
    logits = torch.empty((rows, vocab_local), dtype=x.dtype, device=dev)
    part = torch.empty((num_n, rows, 2), dtype=torch.float32, device=dev)
    target = torch.empty(rows, dtype=torch.float32, device=dev)
    labels = labels.contiguous()
    err = K.status_word(dev)
    ws = workspace(pctx, dev) if pctx.tp_size > 1 else None
    if gather and tp > 1:
        ws.ensure(rows * hidden * 2, 0, 2 * 8 * rows * 16)
        X = torch.empty((rows, hidden), dtype=x.dtype, device=dev)
        K.C.fused_tp_gemm(2, x, w, False, logits, ws.ptrs, pctx.tp_rank, rows, ws.gather_off, ws.recv_off,
                          ws.flags_off, ws.next_epoch(), False, err, TIMEOUT_S, save_out=X, labels=labels,
                          vocab_start=vocab_start, ce_part=part, ce_target=target)
    else:
        # Local GEMM (the kernel with a group of one: no workspace is touched).
        X = x
        K.C.fused_tp_gemm(2, x, w, False, logits, [0], 0, rows, 0, 0, 0, 1, False, err, TIMEOUT_S,
                          labels=labels, vocab_start=vocab_start, ce_part=part, ce_target=target)
    K._count()
    loss = torch.empty(rows, dtype=torch.float32, device=dev)
    gmax = torch.empty_like(loss)
    gsum = torch.empty_like(loss)
    if ws is not None:
        ws.ensure(0, 0, 2 * 8 * rows * 16)
        K.C.ce_merge(part, target, labels, vocab_start, vocab_end, ws.ptrs, pctx.tp_rank, ws.ce_off, ws.flags_off,
                     ws.next_ce_epoch(), err, TIMEOUT_S, loss, gmax, gsum)
    else:
        K.C.ce_merge(part, target, labels, vocab_start, vocab_end, [], 0, 0, 0, 1, err, TIMEOUT_S, loss,
                     gmax, gsum)
    K._count()
    return loss, logits, gmax, gsum, X
