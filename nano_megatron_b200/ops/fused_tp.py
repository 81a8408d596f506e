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

``op(w)`` is ``w`` (``[K, N]``) or, with ``transpose_b=True``, ``w^T`` for
``w [N, K]``. A gathered tensor returned by ``all_gather_matmul(...,
return_gathered=True)`` is a view of the workspace and is valid only until the
next fused call on this TP group.

Parity: replaces the NCCL collectives of ``nano_megatron/mappings.py:43-80``
(same values: concatenation in TP-rank order, SUM reduce-scatter).
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
    """Symmetric workspace of one TP group: flags | gather buffer | recv buffer."""

    def __init__(self, pctx: ParallelContext, device: torch.device):
        self.pctx = pctx
        self.device = device
        self.epoch = 0
        self.buf = None
        self.handle = None
        self.gather_bytes = 0
        self.recv_bytes = 0
        self.flag_bytes = _round(K.C.fused_tp_flag_bytes())

    def ensure(self, gather_bytes: int, recv_bytes: int) -> None:
        if gather_bytes <= self.gather_bytes and recv_bytes <= self.recv_bytes:
            return
        import torch.distributed._symmetric_memory as symm
        gather_bytes = max(_round(gather_bytes), self.gather_bytes)
        recv_bytes = max(_round(recv_bytes), self.recv_bytes)
        if self.buf is not None:
            # Every rank's kernels on the old buffer must be finished before it goes.
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.pctx.tp_group)
        total = self.flag_bytes + gather_bytes + recv_bytes
        buf = symm.empty(total, dtype=torch.uint8, device=self.device)
        buf.zero_()
        handle = symm.rendezvous(buf, self.pctx.tp_group)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.pctx.tp_group)
        self.buf, self.handle = buf, handle
        self.ptrs = [int(p) for p in handle.buffer_ptrs]
        self.gather_bytes, self.recv_bytes = gather_bytes, recv_bytes
        self.flags_off = 0
        self.gather_off = self.flag_bytes
        self.recv_off = self.flag_bytes + gather_bytes

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

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
                      return_gathered: bool = False):
    """``AG(x_local) @ op(w)``; with ``return_gathered`` also the gathered input."""
    x_local = x_local.contiguous()
    m_chunk, k = x_local.shape
    rows = m_chunk * pctx.tp_size
    n = w.shape[0] if transpose_b else w.shape[1]
    ws = workspace(pctx, x_local.device)
    ws.ensure(rows * k * 2, 0)
    out = torch.empty((rows, n), dtype=x_local.dtype, device=x_local.device)
    K.C.fused_tp_gemm(0, x_local, w, not transpose_b, out, ws.ptrs, pctx.tp_rank, rows, ws.gather_off,
                      ws.recv_off, ws.flags_off, ws.next_epoch(), return_gathered,
                      K.status_word(x_local.device), TIMEOUT_S)
    K._count()
    if return_gathered:
        return ws.gathered(rows, k), out
    return out


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


def all_gather(x_local, pctx: ParallelContext):
    """Plain sequence all-gather (NCCL), for the weight-gradient input."""
    out = torch.empty((x_local.shape[0] * pctx.tp_size, *x_local.shape[1:]), dtype=x_local.dtype,
                      device=x_local.device)
    dist.all_gather_into_tensor(out, x_local.contiguous(), group=pctx.tp_group)
    return out
