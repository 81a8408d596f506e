"""Token input for training: a memory-mapped pre-tokenized file and the
synthetic uniform generator.

A token file is a headerless array of native-endian ``uint16`` or ``uint32``
ids. :class:`TokenFile` owns the mapping and a fingerprint of the file
(resolved path, byte size, modification time) so a resumed run can tell that
it is reading the same bytes. :class:`TokenStream` turns the file into
next-token windows for one data-parallel rank.

Window arithmetic (the same positions as ``nano_megatron/data.py:86-92``,
so a cursor means the same training position in both implementations): one
call with batch ``B`` and sequence ``S`` covers ``n = B*S`` positions; DP
rank ``r`` of ``d`` reads the ``n + 1`` tokens that start at
``cursor + r*n`` (inputs are the first ``n``, labels the last ``n``), and
every rank then advances ``cursor`` by ``d*n``. Positions wrap modulo the
file length. The cursor only grows; it is the whole resumable state.

Reads are one or two contiguous slices of the mapping (two when the window
crosses the end of the file), so a window costs one copy of ``n + 1`` ids and
no index array. ``next_batch(pin=True)`` returns page-locked tensors for an
asynchronous host-to-device copy.
"""

from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import torch

# token width name -> numpy dtype of one id in the file (native byte order)
TOKEN_WIDTHS = {"uint16": np.dtype("=u2"), "uint32": np.dtype("=u4")}


class TokenFile:
    """Read-only mapping of a token file plus its fingerprint."""

    def __init__(self, path: str | os.PathLike, width: str):
        if width not in TOKEN_WIDTHS:
            raise ValueError(f"token width {width!r} is not supported; use one of "
                             f"{', '.join(sorted(TOKEN_WIDTHS))}")
        self.path = Path(path)
        info = self.path.stat()
        item = TOKEN_WIDTHS[width].itemsize
        whole, stray = divmod(info.st_size, item)
        if stray:
            raise ValueError(f"{self.path}: {info.st_size} bytes is not a whole number of "
                             f"{item}-byte {width} ids ({stray} stray bytes)")
        if whole < 2:
            raise ValueError(f"{self.path}: {whole} token(s) cannot form an (input, label) pair")
        self.width = width
        self.length = whole
        self.fingerprint = {"path": str(self.path.resolve()), "bytes": int(info.st_size),
                            "mtime_ns": int(info.st_mtime_ns)}
        self._ids = np.memmap(self.path, dtype=TOKEN_WIDTHS[width], mode="r", shape=(whole,))

    def read_cyclic(self, start: int, count: int, out: np.ndarray) -> None:
        """Write ids ``start, start+1, ... (mod length)`` into ``out[:count]``."""
        ids, length = self._ids, self.length
        pos = start % length
        filled = 0
        while filled < count:  # at most two passes unless the window exceeds the file
            take = min(count - filled, length - pos)
            out[filled:filled + take] = ids[pos:pos + take]
            filled += take
            pos = 0


class TokenStream:
    """Next-token ``(inputs, labels)`` windows of one data-parallel rank."""

    def __init__(self, path: str | os.PathLike, *, dtype: str, seq_len: int,
                 dp_rank: int = 0, dp_size: int = 1) -> None:
        if seq_len < 1:
            raise ValueError(f"TokenStream: seq_len={seq_len}; a window needs at least one position")
        if dp_size < 1 or not 0 <= dp_rank < dp_size:
            raise ValueError(f"TokenStream: data-parallel rank {dp_rank} does not exist in a "
                             f"group of {dp_size}")
        self.file = TokenFile(path, dtype)
        self.path, self.dtype, self.seq_len = self.file.path, dtype, seq_len
        self.dp_rank, self.dp_size = dp_rank, dp_size
        self.cursor = 0

    @property
    def num_tokens(self) -> int:
        return self.file.length

    def _layout(self) -> dict:
        return {"dtype": self.dtype, "seq_len": self.seq_len, "dp_rank": self.dp_rank,
                "dp_size": self.dp_size}

    def next_batch(self, batch_size: int, *, pin: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
        """``(input_ids, labels)`` as int64 ``[batch_size, seq_len]`` and advance the cursor."""
        if batch_size < 1:
            raise ValueError(f"TokenStream.next_batch: batch_size={batch_size} must be >= 1")
        n = batch_size * self.seq_len
        window = torch.empty(n + 1, dtype=torch.int64, pin_memory=pin)
        self.file.read_cyclic(self.cursor + self.dp_rank * n, n + 1, window.numpy())
        self.cursor += self.dp_size * n
        return (window[:n].view(batch_size, self.seq_len),
                window[1:].view(batch_size, self.seq_len))

    def state_dict(self) -> dict:
        return {"cursor": self.cursor, "layout": self._layout(), "file": dict(self.file.fingerprint)}

    def load_state_dict(self, state: dict) -> None:
        cursor = state.get("cursor")
        if type(cursor) is not int or cursor < 0:
            raise ValueError(f"TokenStream: saved cursor {cursor!r} is not a non-negative int")
        differences = [f"{what} {key}: saved {saved.get(key)!r}, now {now[key]!r}"
                       for what, saved, now in (("layout", state.get("layout") or {}, self._layout()),
                                                ("file", state.get("file") or {}, self.file.fingerprint))
                       for key in now if saved.get(key) != now[key]]
        if differences:
            raise ValueError("TokenStream: the saved position belongs to a different stream ("
                             + "; ".join(differences) + ")")
        self.cursor = cursor


def synthetic_batches(config, micro_bs: int, num_microbatches: int, step: int,
                      data_parallel_rank: int = 0):
    """Uniform random ``(inputs, labels)`` microbatches for one step of one DP rank.

    The CPU generator is seeded with ``1234 + 100003 * step + dp_rank`` and
    draws inputs, then labels, per microbatch (``nano_megatron/train.py:29-39``),
    so every pipeline stage and TP rank of a DP lane sees the same tokens and
    the two implementations train on identical data.
    """
    gen = torch.Generator().manual_seed(1234 + 100_003 * step + data_parallel_rank)
    shape = (micro_bs, config.seq_len)
    batches = []
    for _ in range(num_microbatches):
        inputs = torch.randint(0, config.vocab_size, shape, generator=gen)
        labels = torch.randint(0, config.vocab_size, shape, generator=gen)
        batches.append((inputs, labels))
    return batches
