"""The cross-entropy gradient kernel launches one grid row per token (at most
65535 per launch). Longer inputs run as launches over consecutive row blocks
of the same tensors; shorter ones as one launch on the tensors as given. The
launch plan is checked on the host with a stand-in for the kernel."""

import pytest
import torch

K = pytest.importorskip("nano_megatron_b200.ops.cuda", reason="the extension is not built",
                        exc_type=ImportError)


class Recorder:
    def __init__(self):
        self.calls = []

    def ce_grad(self, logits, target, gmax, gsum, scale, inv_n, d, vstart):
        n = logits.shape[0]
        assert n <= 65535
        assert target.shape[0] == gmax.shape[0] == gsum.shape[0] == d.shape[0] == n
        assert all(t.is_contiguous() for t in (target, gmax, gsum, d)) and logits.stride(1) == 1
        self.calls.append((logits.data_ptr(), d.data_ptr(), n))


@pytest.mark.parametrize("rows", [1, 8192, 65535, 65536, 100000])
def test_row_blocks_cover_every_row_once(monkeypatch, rows):
    rec = Recorder()
    monkeypatch.setattr(K, "C", rec)
    vocab = 16
    logits = torch.zeros(rows, vocab, dtype=torch.bfloat16)
    d = torch.empty_like(logits)
    target = torch.zeros(rows, dtype=torch.int64)
    g = torch.zeros(rows)
    K._ce_grad_launch(logits, target, g, g.clone(), torch.ones(1), d, 0)
    if rows <= 65535:
        assert rec.calls == [(logits.data_ptr(), d.data_ptr(), rows)]
        return
    row_bytes = vocab * logits.element_size()
    covered = 0
    for lp, dp, n in rec.calls:
        assert lp == logits.data_ptr() + covered * row_bytes and dp == d.data_ptr() + covered * row_bytes
        covered += n
    assert covered == rows and len(rec.calls) == -(-rows // 32768)
