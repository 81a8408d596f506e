"""Token stream: disjoint DP windows, cursor round trip and wrap, uint32 ids,
input validation."""

import struct

import pytest
import torch

from nano_megatron_b200.utils.data import TokenStream, synthetic_batches
from nano_megatron_b200.models import GPTConfig


def _write(path, values, dtype="uint16"):
    path.write_bytes(struct.pack(f"={len(values)}{ {'uint16': 'H', 'uint32': 'I'}[dtype]}", *values))
    return path


def test_dp_ranks_read_disjoint_windows(tmp_path):
    path = _write(tmp_path / "t.bin", range(40))
    r0 = TokenStream(path, dtype="uint16", seq_len=3, dp_rank=0, dp_size=2)
    r1 = TokenStream(path, dtype="uint16", seq_len=3, dp_rank=1, dp_size=2)
    x0, y0 = r0.next_batch(2)
    x1, y1 = r1.next_batch(2)
    assert x0.flatten().tolist() == list(range(6)) and y0.flatten().tolist() == list(range(1, 7))
    assert x1.flatten().tolist() == list(range(6, 12)) and y1.flatten().tolist() == list(range(7, 13))
    assert r0.cursor == r1.cursor == 12
    assert r0.next_batch(2)[0].flatten().tolist() == list(range(12, 18))
    assert r1.next_batch(2)[0].flatten().tolist() == list(range(18, 24))


def test_cursor_round_trip_and_wrap(tmp_path):
    path = _write(tmp_path / "t.bin", range(10))
    s = TokenStream(path, dtype="uint16", seq_len=3, dp_rank=1, dp_size=2)
    s.next_batch(1)
    saved = s.state_dict()
    expected = s.next_batch(1)
    resumed = TokenStream(path, dtype="uint16", seq_len=3, dp_rank=1, dp_size=2)
    resumed.load_state_dict(saved)
    got = resumed.next_batch(1)
    assert torch.equal(got[0], expected[0]) and torch.equal(got[1], expected[1])
    assert got[0].flatten().tolist() == [9, 0, 1] and got[1].flatten().tolist() == [0, 1, 2]


def test_uint32_not_truncated(tmp_path):
    path = _write(tmp_path / "t.bin", [0, 70_000, 80_000, 90_000], "uint32")
    x, y = TokenStream(path, dtype="uint32", seq_len=2).next_batch(1)
    assert x.dtype == y.dtype == torch.int64
    assert x.tolist() == [[0, 70_000]] and y.tolist() == [[70_000, 80_000]]


def test_validation(tmp_path):
    path = _write(tmp_path / "t.bin", range(4))
    with pytest.raises(ValueError, match="dtype"):
        TokenStream(path, dtype="int64", seq_len=2)
    with pytest.raises(ValueError, match="dp_rank"):
        TokenStream(path, dtype="uint16", seq_len=2, dp_rank=2, dp_size=2)
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"abc")
    with pytest.raises(ValueError, match="not divisible"):
        TokenStream(bad, dtype="uint16", seq_len=2)
    s = TokenStream(path, dtype="uint16", seq_len=2)
    st = s.state_dict()
    st["cursor"] = -1
    with pytest.raises(ValueError, match="cursor"):
        s.load_state_dict(st)
    st = s.state_dict()
    st["seq_len"] = 4
    with pytest.raises(ValueError, match="configuration mismatch"):
        s.load_state_dict(st)


def test_synthetic_batches_seeded_per_step_and_dp_rank():
    cfg = GPTConfig(vocab_size=50, seq_len=6)
    a = synthetic_batches(cfg, 2, 3, step=5, data_parallel_rank=1)
    b = synthetic_batches(cfg, 2, 3, step=5, data_parallel_rank=1)
    c = synthetic_batches(cfg, 2, 3, step=5, data_parallel_rank=0)
    assert all(torch.equal(x1, x2) and torch.equal(y1, y2) for (x1, y1), (x2, y2) in zip(a, b))
    assert not torch.equal(a[0][0], c[0][0])
    gen = torch.Generator().manual_seed(1234 + 100_003 * 5 + 1)
    assert torch.equal(a[0][0], torch.randint(0, 50, (2, 6), generator=gen))
