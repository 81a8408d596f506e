"""Token input: windows tile the file across DP ranks and steps, labels are the
inputs shifted by one, reads wrap cyclically, the position survives a
save/load and is refused for a different stream, wide ids stay exact, and the
synthetic generator follows its seed formula."""

import numpy as np
import pytest
import torch

from nano_megatron_b200.models import GPTConfig
from nano_megatron_b200.utils.data import TokenFile, TokenStream, synthetic_batches


def _token_file(path, ids, width="uint16"):
    np.asarray(ids, dtype={"uint16": "=u2", "uint32": "=u4"}[width]).tofile(path)
    return path


@pytest.fixture
def primes_file(tmp_path):
    # 997 ids with no repeats inside any short window: a wrong offset shows up
    ids = [(i * 37 + 11) % 997 for i in range(997)]
    return _token_file(tmp_path / "ids.bin", ids), np.array(ids)


@pytest.mark.parametrize("dp_size", [1, 3])
def test_rank_windows_tile_the_stream_in_order(primes_file, dp_size):
    path, ids = primes_file
    seq, batch, steps = 5, 4, 6
    streams = [TokenStream(path, dtype="uint16", seq_len=seq, dp_rank=r, dp_size=dp_size)
               for r in range(dp_size)]
    consumed = []
    for _ in range(steps):
        for s in streams:
            x, _ = s.next_batch(batch)
            assert x.shape == (batch, seq) and x.dtype == torch.int64
            consumed.extend(x.flatten().tolist())
    n = len(consumed)
    assert consumed == [int(ids[i % len(ids)]) for i in range(n)]
    assert all(s.cursor == steps * dp_size * batch * seq for s in streams)


def test_labels_are_inputs_shifted_by_one(primes_file):
    path, ids = primes_file
    s = TokenStream(path, dtype="uint16", seq_len=7, dp_rank=1, dp_size=2)
    for _ in range(40):  # crosses the end of the file several times
        start = s.cursor + 1 * 3 * 7
        x, y = s.next_batch(3)
        flat_x, flat_y = x.flatten().numpy(), y.flatten().numpy()
        expect = ids[(np.arange(22) + start) % len(ids)]
        assert (flat_x == expect[:-1]).all() and (flat_y == expect[1:]).all()


def test_window_longer_than_the_file_wraps_repeatedly(tmp_path):
    path = _token_file(tmp_path / "short.bin", [5, 6, 7])
    x, y = TokenStream(path, dtype="uint16", seq_len=4).next_batch(2)
    assert x.flatten().tolist() == [5, 6, 7, 5, 6, 7, 5, 6]
    assert y.flatten().tolist() == [6, 7, 5, 6, 7, 5, 6, 7]
    out = np.zeros(7, dtype=np.int64)
    TokenFile(path, "uint16").read_cyclic(2, 7, out)
    assert out.tolist() == [7, 5, 6, 7, 5, 6, 7]


def test_resume_continues_exactly_and_rejects_another_stream(primes_file, tmp_path):
    path, _ = primes_file
    a = TokenStream(path, dtype="uint16", seq_len=6, dp_rank=0, dp_size=2)
    for _ in range(9):
        a.next_batch(5)
    saved = a.state_dict()
    following = [a.next_batch(5) for _ in range(3)]
    b = TokenStream(path, dtype="uint16", seq_len=6, dp_rank=0, dp_size=2)
    b.load_state_dict(saved)
    for (xa, ya), (xb, yb) in zip(following, [b.next_batch(5) for _ in range(3)]):
        assert torch.equal(xa, xb) and torch.equal(ya, yb)

    other_rank = TokenStream(path, dtype="uint16", seq_len=6, dp_rank=1, dp_size=2)
    with pytest.raises(ValueError, match="dp_rank"):
        other_rank.load_state_dict(saved)
    grown = _token_file(tmp_path / "grown.bin", list(range(998)))
    with pytest.raises(ValueError, match="bytes"):
        TokenStream(grown, dtype="uint16", seq_len=6, dp_rank=0, dp_size=2).load_state_dict(
            {**saved, "file": {**saved["file"], "path": str(grown.resolve())}})
    for bad in (-3, 2.0, True, None):
        with pytest.raises(ValueError, match="cursor"):
            b.load_state_dict({**saved, "cursor": bad})


def test_wide_ids_are_kept_exactly(tmp_path):
    ids = [65_535, 65_536, 128_255, 4_000_000_000, 1]
    path = _token_file(tmp_path / "wide.bin", ids, "uint32")
    x, y = TokenStream(path, dtype="uint32", seq_len=4).next_batch(1)
    assert x.tolist() == [ids[:4]] and y.tolist() == [ids[1:]]


def test_unusable_inputs_are_refused(tmp_path):
    path = _token_file(tmp_path / "ok.bin", range(8))
    (tmp_path / "odd.bin").write_bytes(bytes(9))
    _token_file(tmp_path / "one.bin", [3])
    cases = [
        (dict(path=path, dtype="int32", seq_len=2), "width"),
        (dict(path=tmp_path / "odd.bin", dtype="uint16", seq_len=2), "stray"),
        (dict(path=tmp_path / "one.bin", dtype="uint16", seq_len=1), "pair"),
        (dict(path=path, dtype="uint16", seq_len=0), "seq_len"),
        (dict(path=path, dtype="uint16", seq_len=2, dp_rank=3, dp_size=3), "rank 3"),
    ]
    for kwargs, message in cases:
        with pytest.raises(ValueError, match=message):
            TokenStream(kwargs.pop("path"), **kwargs)
    with pytest.raises(ValueError, match="batch_size"):
        TokenStream(path, dtype="uint16", seq_len=2).next_batch(0)


def test_synthetic_generator_seed_formula():
    cfg = GPTConfig(vocab_size=321, seq_len=9)
    step, lane = 17, 3
    batches = synthetic_batches(cfg, 2, 4, step=step, data_parallel_rank=lane)
    gen = torch.Generator().manual_seed(1234 + 100_003 * step + lane)
    for inputs, labels in batches:
        assert torch.equal(inputs, torch.randint(0, 321, (2, 9), generator=gen))
        assert torch.equal(labels, torch.randint(0, 321, (2, 9), generator=gen))
    neighbour = synthetic_batches(cfg, 2, 4, step=step, data_parallel_rank=lane + 1)
    assert not torch.equal(batches[0][0], neighbour[0][0])
