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

Inputs may have any number of leading dims; with sequence parallelism the
sequence is dim 0 (sequence-first layout, see ``parallel/mappings.py``).
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


class ColumnParallelLinear(nn.Module):
    """``y = x @ A`` with ``A = [A_1 | ... | A_tp]`` split along the output dim."""

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
        """``reduce_input_grad`` applies f; ``sequence_parallel`` all-gathers dim 0 first."""
        mode = "ag" if sequence_parallel else ("f" if reduce_input_grad else "none")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        y = column_linear(x2, WeightRef.of(self.weight), self.ctx, mode, _dtype_of(x))
        if sequence_parallel:
            lead = (lead[0] * self.ctx.tp_size, *lead[1:]) if len(lead) else lead
        y = y.view(*lead, self.out_features_local)
        return y + self.bias.to(y.dtype) if self.bias is not None else y


class RowParallelLinear(nn.Module):
    """``y = x @ A`` with ``A`` split along the input dim and ``x`` sharded to match."""

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
        mode = "rs" if sequence_parallel else ("g" if reduce_output else "none")
        lead = x.shape[:-1]
        y = row_linear(x.reshape(-1, x.shape[-1]), WeightRef.of(self.weight), self.ctx, mode,
                       _dtype_of(x))
        if sequence_parallel and len(lead):
            lead = (lead[0] // self.ctx.tp_size, *lead[1:])
        y = y.view(*lead, self.out_features)
        return y + self.bias.to(y.dtype) if self.bias is not None else y


class VocabParallelEmbedding(nn.Module):
    """Embedding table sharded along the vocabulary across the TP group."""

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
        """``input_ids`` of any shape; with SP it must be sequence-first ``[S, ...]``."""
        if not input_ids.is_cuda:
            # CUDA checks bounds inside the kernel (device error flag, no sync).
            if torch.any(input_ids < 0) or torch.any(input_ids >= self.num_embeddings):
                raise ValueError("input token id is outside the model vocabulary")
        lead = input_ids.shape
        mode = "rs" if sequence_parallel else "ar"
        y = vocab_embedding(input_ids.reshape(-1), WeightRef.of(self.weight), self.ctx, mode,
                            self.vocab_start, self.vocab_end, out_dtype or self.weight.dtype)
        if sequence_parallel and self.ctx.tp_size > 1:
            lead = (lead[0] // self.ctx.tp_size, *lead[1:])
        return y.view(*lead, -1)


class RMSNorm(nn.Module):
    """Root-mean-square norm; replicated across TP (every rank sees the same input)."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        lead = x.shape[:-1]
        return rms_norm(x.reshape(-1, x.shape[-1]), self.weight, self.eps).view(*lead, x.shape[-1])
