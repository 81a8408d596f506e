"""Autograd-aware tensor- and sequence-parallel collectives.

Four conjugate pairs; each backward is the adjoint of its forward:

==========================================  =====================  =====================
function                                    forward                backward
==========================================  =====================  =====================
``copy_to_tensor_parallel_region`` (f)      identity               all-reduce (SUM)
``reduce_from_tensor_parallel_region`` (g)  all-reduce (SUM)       identity
``gather_from_sequence_parallel_region``    all-gather along seq   reduce-scatter (SUM)
``reduce_scatter_to_sequence_parallel_...`` reduce-scatter (SUM)   all-gather along seq
==========================================  =====================  =====================

Inside a stage, activations in this framework are token rows in
sequence-major order (``[s*b, H]``), so a sequence shard is one contiguous slab and the
model's own gather/scatter (``all_gather_sequence`` and
``reduce_scatter_sequence``, sequence on dim 0 by default) need no transposes.
The four public functions keep the reference's batch-first convention: the
sequence is dim 1 of ``[b, s, ...]`` unless ``seq_dim=0`` is passed for a
sequence-first tensor.

These are the generic (NCCL / Gloo) paths. On CUDA with tensor parallelism the
linear layers use fused all-gather->GEMM and GEMM->reduce-scatter kernels
instead (``nano_megatron_b200.ops.fused_tp``), which compute the same values.

Parity: ``nano_megatron/mappings.py:29-152``.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .context import ParallelContext


def _all_reduce(tensor: torch.Tensor, group, world_size: int) -> torch.Tensor:
    """In-place SUM all-reduce; a no-op for a group of one (tests patch this)."""
    if world_size == 1:
        return tensor
    dist.all_reduce(tensor, group=group)
    return tensor


def _to_seq_first(tensor: torch.Tensor, seq_dim: int) -> torch.Tensor:
    if tensor.ndim < 2 and seq_dim != 0:
        raise ValueError(f"sequence-parallel tensor needs at least 2 dims, got {tuple(tensor.shape)}")
    return tensor if seq_dim == 0 else tensor.transpose(0, seq_dim)


def all_gather_sequence(tensor: torch.Tensor, group, world_size: int, seq_dim: int = 0) -> torch.Tensor:
    """Concatenate every rank's sequence shard in TP-rank order."""
    if world_size == 1:
        return tensor
    if tensor.ndim < 1:
        raise ValueError("sequence-parallel tensor needs at least 1 dim")
    local = _to_seq_first(tensor, seq_dim).contiguous()
    out = torch.empty((local.shape[0] * world_size, *local.shape[1:]),
                      dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local, group=group)
    return out if seq_dim == 0 else out.transpose(0, seq_dim).contiguous()


def reduce_scatter_sequence(tensor: torch.Tensor, group, world_size: int, seq_dim: int = 0) -> torch.Tensor:
    """SUM full-sequence partials across ranks; keep this rank's sequence shard."""
    if world_size == 1:
        return tensor
    full = _to_seq_first(tensor, seq_dim)
    if full.shape[0] % world_size:
        raise ValueError(
            f"sequence length {full.shape[0]} is not divisible by TP size {world_size}")
    full = full.contiguous()
    out = torch.empty((full.shape[0] // world_size, *full.shape[1:]),
                      dtype=full.dtype, device=full.device)
    dist.reduce_scatter_tensor(out, full, op=dist.ReduceOp.SUM, group=group)
    return out if seq_dim == 0 else out.transpose(0, seq_dim).contiguous()


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, world_size):
        ctx.group, ctx.world_size = group, world_size
        return x.view_as(x)

    @staticmethod
    def backward(ctx, grad):
        return _all_reduce(grad.contiguous(), ctx.group, ctx.world_size), None, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, world_size):
        if world_size == 1:
            return x.view_as(x)
        return _all_reduce(x.clone(memory_format=torch.contiguous_format), group, world_size)

    @staticmethod
    def backward(ctx, grad):
        return grad, None, None


class _GatherSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, world_size, seq_dim):
        ctx.group, ctx.world_size, ctx.seq_dim = group, world_size, seq_dim
        return all_gather_sequence(x, group, world_size, seq_dim)

    @staticmethod
    def backward(ctx, grad):
        return reduce_scatter_sequence(grad, ctx.group, ctx.world_size, ctx.seq_dim), None, None, None


class _ReduceScatterSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, world_size, seq_dim):
        ctx.group, ctx.world_size, ctx.seq_dim = group, world_size, seq_dim
        return reduce_scatter_sequence(x, group, world_size, seq_dim)

    @staticmethod
    def backward(ctx, grad):
        return all_gather_sequence(grad, ctx.group, ctx.world_size, ctx.seq_dim), None, None, None


def copy_to_tensor_parallel_region(x: torch.Tensor, ctx: ParallelContext) -> torch.Tensor:
    return _CopyToTP.apply(x, ctx.tp_group, ctx.tp_size)


def reduce_from_tensor_parallel_region(x: torch.Tensor, ctx: ParallelContext) -> torch.Tensor:
    return _ReduceFromTP.apply(x, ctx.tp_group, ctx.tp_size)


def gather_from_sequence_parallel_region(x: torch.Tensor, ctx: ParallelContext,
                                         seq_dim: int = 1) -> torch.Tensor:
    """All-gather the sequence shards (dim ``seq_dim``, 1 for batch-first ``[b, s, ...]``)."""
    return _GatherSeq.apply(x, ctx.tp_group, ctx.tp_size, seq_dim)


def reduce_scatter_to_sequence_parallel_region(x: torch.Tensor, ctx: ParallelContext,
                                               seq_dim: int = 1) -> torch.Tensor:
    """SUM the full-sequence partials and keep this rank's shard of dim ``seq_dim``."""
    return _ReduceScatterSeq.apply(x, ctx.tp_group, ctx.tp_size, seq_dim)
