"""Tensor-parallel layers and RMSNorm.

Weight layouts, shapes, init and the ``tensor_parallel_sharded`` tag follow
``nano_megatron/tp_layers.py:34-132`` and ``model.py:65-75``:

* ``ColumnParallelLinear``: weight ``[in, out/tp]`` (output features sharded),
  optional sharded bias;
* ``RowParallelLinear``: weight ``[in/tp, out]``, optional replicated bias added
  after the reduction;
* ``VocabParallelEmbedding``: table ``[V/tp, H]``, rows outside this rank's
  vocabulary slice contribute zeros and the reduction fills them in;
* ``RMSNorm``: eps 1e-6, fp32 statistics, replicated (not tagged sharded).

Inputs may have any number of leading dims. With sequence parallelism a
tensor of three or more dims is batch-first ``[b, s, ...]`` as in the
reference, and the sequence collective acts on dim 1; a 2-D ``[T, H]`` input
is a block of token rows whose sequence shard is a contiguous row range (the
model's own sequence-first layout, see ``parallel/mappings.py``).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from ..parallel.context import ParallelContext
from .config import divide
from .functional import (WeightRef, column_linear, rms_norm, row_linear,
                         vocab_embedding)


def _dtype_of(x: torch.Tensor) -> torch.dtype:
    return x.dtype if x.is_floating_point() else torch.float32


def _sequence_rows(x: torch.Tensor, sequence_parallel: bool, min_dims: int):
    """``x`` with the sequence on dim 0, and whether it was batch-first.

    Batch-first inputs (``min_dims`` or more dims) under sequence parallelism
    are transposed so that the flattened rows are sequence-major and a
    sequence shard is a contiguous row range."""
    if sequence_parallel and x.dim() >= min_dims:
        return x.transpose(0, 1), True
    return x, False


def _check_sequence(length: int, ctx: ParallelContext) -> None:
    if length % ctx.tp_size:
        raise ValueError(f"sequence length {length} is not divisible by TP size {ctx.tp_size}")


class ColumnParallelLinear(nn.Module):
    """``y = x @ A`` with ``A = [A_1 | ... | A_tp]`` split along the output dim.

    Parity: ``nano_megatron/tp_layers.py:34-61`` (the ``sequence_parallel``
    all-gather is the reference's outer ``gather_from_sequence_parallel_region``,
    ``model.py:113-114``, folded into the layer so CUDA can fuse it into the GEMM).
    """

    def __init__(self, in_features: int, out_features: int, ctx: ParallelContext,
                 bias: bool = True, init_std: float = 0.02):
        super().__init__()
        self.ctx = ctx
        self.in_features = in_features
        self.out_features_local = divide(out_features, ctx.tp_size)
        self.weight = nn.Parameter(torch.empty(in_features, self.out_features_local))
        self.bias = nn.Parameter(torch.zeros(self.out_features_local)) if bias else None
        self.weight.tensor_parallel_sharded = True
        if self.bias is not None:
            self.bias.tensor_parallel_sharded = True
        nn.init.normal_(self.weight, std=init_std)

    def forward(self, x, *, reduce_input_grad: bool = True, sequence_parallel: bool = False):
        """``reduce_input_grad`` applies f; ``sequence_parallel`` (an extension)
        all-gathers the sequence first: dim 1 of a batch-first ``[b, s, H]``,
        the rows of a 2-D ``[T, H]``."""
        mode = "ag" if sequence_parallel else ("f" if reduce_input_grad else "none")
        xs, batch_first = _sequence_rows(x, sequence_parallel, 3)
        lead = xs.shape[:-1]
        y = column_linear(xs.reshape(-1, xs.shape[-1]), WeightRef.of(self.weight), self.ctx, mode,
                          _dtype_of(x))
        if sequence_parallel:
            lead = (lead[0] * self.ctx.tp_size, *lead[1:]) if len(lead) else lead
        y = y.view(*lead, self.out_features_local)
        if batch_first:
            y = y.transpose(0, 1).contiguous()
        return y + self.bias.to(y.dtype) if self.bias is not None else y


class RowParallelLinear(nn.Module):
    """``y = x @ A`` with ``A`` split along the input dim and ``x`` sharded to match.

    Parity: ``nano_megatron/tp_layers.py:64-88`` (reduce-scatter under sequence
    parallelism, all-reduce otherwise; the bias after the reduction).
    """

    def __init__(self, in_features: int, out_features: int, ctx: ParallelContext,
                 bias: bool = True, init_std: float = 0.02):
        super().__init__()
        self.ctx = ctx
        self.out_features = out_features
        self.in_features_local = divide(in_features, ctx.tp_size)
        self.weight = nn.Parameter(torch.empty(self.in_features_local, out_features))
        # Replicated bias, added after the reduction (adding it before would
        # count it tp times).
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None
        self.weight.tensor_parallel_sharded = True
        nn.init.normal_(self.weight, std=init_std)

    def forward(self, x, *, sequence_parallel: bool = False, reduce_output: bool = True):
        """All-reduce (g) the partial products, or with ``sequence_parallel``
        reduce-scatter them along the sequence: dim 1 of a batch-first
        ``[b, S, H/tp]``, the rows of a 2-D ``[T, H/tp]``. ``reduce_output=False``
        (an extension) returns the partial products."""
        mode = "rs" if sequence_parallel else ("g" if reduce_output else "none")
        xs, batch_first = _sequence_rows(x, sequence_parallel, 3)
        lead = xs.shape[:-1]
        if sequence_parallel and len(lead):
            _check_sequence(lead[0], self.ctx)
        y = row_linear(xs.reshape(-1, xs.shape[-1]), WeightRef.of(self.weight), self.ctx, mode,
                       _dtype_of(x))
        if sequence_parallel and len(lead):
            lead = (lead[0] // self.ctx.tp_size, *lead[1:])
        y = y.view(*lead, self.out_features)
        if batch_first:
            y = y.transpose(0, 1).contiguous()
        return y + self.bias.to(y.dtype) if self.bias is not None else y


class VocabParallelEmbedding(nn.Module):
    """Embedding table sharded along the vocabulary across the TP group.

    Parity: ``nano_megatron/tp_layers.py:91-132``; the id bounds check runs on
    the device on CUDA instead of on the host (``:113-115``).
    """

    def __init__(self, num_embeddings: int, embedding_dim: int, ctx: ParallelContext,
                 init_std: float = 0.02):
        super().__init__()
        self.ctx = ctx
        per_partition = divide(num_embeddings, ctx.tp_size)
        self.num_embeddings = num_embeddings
        self.vocab_start = ctx.tp_rank * per_partition
        self.vocab_end = self.vocab_start + per_partition
        self.weight = nn.Parameter(torch.empty(per_partition, embedding_dim))
        self.weight.tensor_parallel_sharded = True
        nn.init.normal_(self.weight, std=init_std)

    def forward(self, input_ids, *, sequence_parallel: bool = False,
                out_dtype: torch.dtype | None = None):
        """``input_ids [b, S]`` -> ``[b, S, H]``, or ``[b, S/tp, H]`` with
        ``sequence_parallel`` (reduce-scattered along the sequence). Ids of
        other shapes work too; 1-D ids are token rows, scattered by row range."""
        ids, batch_first = _sequence_rows(input_ids, sequence_parallel, 2)
        lead = ids.shape
        if sequence_parallel and self.ctx.tp_size > 1:
            _check_sequence(lead[0], self.ctx)
            lead = (lead[0] // self.ctx.tp_size, *lead[1:])
        y = self.embed_rows(ids.reshape(-1), sequence_parallel=sequence_parallel, out_dtype=out_dtype)
        y = y.view(*lead, -1)
        return y.transpose(0, 1).contiguous() if batch_first else y

    def embed_rows(self, ids: torch.Tensor, *, sequence_parallel: bool = False,
                   out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """1-D ids in sequence-major order -> rows ``[T, H]`` (``[T/tp, H]``, this
        rank's row range, with ``sequence_parallel``)."""
        if not ids.is_cuda:
            # CUDA checks bounds inside the kernel (device error flag, no sync).
            if torch.any(ids < 0) or torch.any(ids >= self.num_embeddings):
                raise ValueError("input token id is outside the model vocabulary")
        mode = "rs" if sequence_parallel else "ar"
        return vocab_embedding(ids, WeightRef.of(self.weight), self.ctx, mode,
                               self.vocab_start, self.vocab_end, out_dtype or self.weight.dtype)


class RMSNorm(nn.Module):
    """Root-mean-square norm; replicated across TP (every rank sees the same input).

    Parity: ``nano_megatron/model.py:65-75`` (fp32 statistics, result cast to
    the input dtype before the weight multiply).
    """

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        lead = x.shape[:-1]
        return rms_norm(x.reshape(-1, x.shape[-1]), self.weight, self.eps).view(*lead, x.shape[-1])
