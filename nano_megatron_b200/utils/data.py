"""Pre-tokenized token streams and the synthetic batch generator.

The file format is a flat, native-endian array of uint16 or uint32 token ids.
DP rank ``r`` of ``d`` reads, for each call, the window starting at
``cursor + r * B * S`` and every rank then advances ``cursor`` by ``d * B * S``;
reads wrap at the end of the file. Only the monotonically growing cursor is
state, so equal cursors mean the same training position on every TP/PP rank.

Parity: ``nano_megatron/data.py:22-123`` (format, window formula, wrap,
state/validation) and ``nano_megatron/train.py:29-39`` (synthetic seeds).
"""

from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import torch

_ITEM = {"uint16": np.dtype("=u2"), "uint32": np.dtype("=u4")}


class TokenStream:
    """Deterministic next-token ``(inputs, labels)`` windows from a memory-mapped file."""

    def __init__(self, path: str | os.PathLike, *, dtype: str, seq_len: int,
                 dp_rank: int = 0, dp_size: int = 1) -> None:
        if dtype not in _ITEM:
            raise ValueError(f"dtype must be one of {sorted(_ITEM)}, got {dtype!r}")
        if seq_len <= 0:
            raise ValueError(f"seq_len must be positive, got {seq_len}")
        if dp_size <= 0:
            raise ValueError(f"dp_size must be positive, got {dp_size}")
        if not 0 <= dp_rank < dp_size:
            raise ValueError(f"dp_rank must be in [0, {dp_size}), got {dp_rank}")
        path = Path(path)
        stat = path.stat()
        item = _ITEM[dtype].itemsize
        if stat.st_size % item:
            raise ValueError(
                f"{path} has {stat.st_size} bytes, not divisible by {dtype} item size {item}")
        count = stat.st_size // item
        if count < 2:
            raise ValueError(f"token stream needs at least 2 tokens, got {count}")
        self.path, self.dtype, self.seq_len = path, dtype, seq_len
        self.dp_rank, self.dp_size = dp_rank, dp_size
        self.cursor = 0
        self._identity = {"path": str(path.resolve()), "size_bytes": stat.st_size,
                          "mtime_ns": stat.st_mtime_ns}
        self._tokens = np.memmap(path, dtype=_ITEM[dtype], mode="r", shape=(count,))

    @property
    def num_tokens(self) -> int:
        return int(self._tokens.shape[0])

    def next_batch(self, batch_size: int) -> tuple[torch.Tensor, torch.Tensor]:
        """``(input_ids, labels)``, each int64 ``[batch_size, seq_len]``."""
        if batch_size <= 0:
            raise ValueError(f"batch_size must be positive, got {batch_size}")
        n = batch_size * self.seq_len
        start = self.cursor + self.dp_rank * n
        idx = (np.arange(n + 1, dtype=np.int64) + start) % self.num_tokens
        window = torch.from_numpy(self._tokens[idx].astype(np.int64))
        self.cursor += self.dp_size * n
        return (window[:-1].view(batch_size, self.seq_len).clone(),
                window[1:].view(batch_size, self.seq_len).clone())

    def state_dict(self) -> dict:
        return {"cursor": self.cursor, "dtype": self.dtype, "seq_len": self.seq_len,
                "dp_rank": self.dp_rank, "dp_size": self.dp_size, "identity": dict(self._identity)}

    def load_state_dict(self, state: dict) -> None:
        expected = {"dtype": self.dtype, "seq_len": self.seq_len, "dp_rank": self.dp_rank,
                    "dp_size": self.dp_size, "identity": self._identity}
        actual = {k: state.get(k) for k in expected}
        if actual != expected:
            raise ValueError(f"token-stream configuration mismatch: saved={actual}, current={expected}")
        cursor = state.get("cursor")
        if isinstance(cursor, bool) or not isinstance(cursor, int) or cursor < 0:
            raise ValueError(f"cursor must be a non-negative integer, got {cursor!r}")
        self.cursor = cursor


def synthetic_batches(config, micro_batch_size: int, num_microbatches: int, step: int,
                      data_parallel_rank: int = 0):
    """Uniform random ``(inputs, labels)`` microbatches, seeded per (step, DP rank).

    Seed ``1234 + 100003 * step + dp_rank``: pipeline stages of one DP lane agree,
    DP replicas differ. Inputs and labels are drawn independently.
    """
    gen = torch.Generator().manual_seed(1234 + 100_003 * step + data_parallel_rank)
    shape = (micro_batch_size, config.seq_len)
    return [(torch.randint(0, config.vocab_size, shape, generator=gen),
             torch.randint(0, config.vocab_size, shape, generator=gen))
            for _ in range(num_microbatches)]
