"""Checkpoint: full restore, atomic failure (host-side fault injection),
topology mismatch rejected before any mutation, incomplete checkpoints."""

import copy
import random
import struct
from unittest import mock

import pytest
import torch
import torch.nn as nn

from nano_megatron_b200.models import GPT, GPTConfig
from nano_megatron_b200.optim import FusedAdamW
from nano_megatron_b200.parallel import ParallelContext
from nano_megatron_b200.utils import checkpoint
from nano_megatron_b200.utils.data import TokenStream

CTX = ParallelContext.single()


def _stream(tmp_path):
    path = tmp_path / "tokens.bin"
    path.write_bytes(struct.pack("=64H", *range(64)))
    return TokenStream(path, dtype="uint16", seq_len=4)


def _state(tmp_path, fused=False):
    torch.manual_seed(11)
    data = _stream(tmp_path)
    if fused:
        model = GPT(GPTConfig(vocab_size=64, n_layer=2, n_head=2, n_embd=16, seq_len=4))
        opt = FusedAdamW(model, lr=0.01)
        x, y = data.next_batch(2)
        model(x, y).backward()
    else:
        model = nn.Linear(2, 2)
        opt = torch.optim.AdamW(model.parameters(), lr=0.01)
        x, y = data.next_batch(2)
        model(x[:, :2].float()).sub(y[:, :2].float()).square().mean().backward()
    opt.step()
    opt.zero_grad()
    return model, opt, data


def _equal(a, b):
    if torch.is_tensor(b):
        assert torch.equal(a, b)
    elif isinstance(b, dict):
        assert a.keys() == b.keys()
        for k in b:
            _equal(a[k], b[k])
    elif isinstance(b, (list, tuple)):
        assert len(a) == len(b)
        for x, y in zip(a, b):
            _equal(x, y)
    else:
        assert a == b


@pytest.mark.parametrize("fused", [False, True])
def test_restores_everything(tmp_path, fused):
    model, opt, data = _state(tmp_path, fused)
    random.seed(23)
    checkpoint.save_checkpoint(tmp_path / "ck", model, opt, CTX, step=7, data=data, extra={"a": 1})
    saved_model = copy.deepcopy(model.state_dict())
    saved_opt = copy.deepcopy(opt.state_dict())
    want_t, want_p, want_b = torch.rand(4), random.random(), data.next_batch(2)
    for p in model.parameters():
        p.data.add_(100)
    opt.param_groups[0]["lr"] = 9.0
    torch.manual_seed(999)
    random.seed(999)
    step, extra = checkpoint.load_checkpoint(tmp_path / "ck", model, opt, CTX, data=data)
    assert step == 7 and extra == {"a": 1}
    _equal(model.state_dict(), saved_model)
    _equal(opt.state_dict(), saved_opt)
    assert torch.equal(torch.rand(4), want_t) and random.random() == want_p
    got_b = data.next_batch(2)
    assert torch.equal(got_b[0], want_b[0]) and torch.equal(got_b[1], want_b[1])
    if fused:  # parameters still view the flat buffer after the load
        base = model.flat_buffers.data
        assert all(base.data_ptr() <= p.data_ptr() < base.data_ptr() + base.numel() * 4
                   for p in model.parameters())


def test_atomic_failure_keeps_previous_shard(tmp_path):
    model, opt, data = _state(tmp_path)
    d = tmp_path / "ck"
    path = checkpoint.save_checkpoint(d, model, opt, CTX, step=3, data=data)
    original = path.read_bytes()

    def partial_write(_obj, tmp):
        tmp.write_bytes(b"partial")
        raise OSError("simulated write failure")

    with mock.patch.object(checkpoint.torch, "save", side_effect=partial_write):
        with pytest.raises(OSError, match="simulated"):
            checkpoint.save_checkpoint(d, model, opt, CTX, step=4, data=data)
    assert path.name == "rank_00000.pt" and path.read_bytes() == original
    assert list(d.glob("*.tmp")) == [] and list(d.glob(".*.tmp")) == []


def test_topology_mismatch_rejected_before_mutation(tmp_path):
    model, opt, data = _state(tmp_path)
    d = tmp_path / "ck"
    path = checkpoint.save_checkpoint(d, model, opt, CTX, step=3, data=data)
    state = torch.load(path, weights_only=False)
    state["topology"]["tp_size"] = 2
    torch.save(state, path)
    before = copy.deepcopy(model.state_dict())
    with pytest.raises(RuntimeError, match="topology mismatch"):
        checkpoint.load_checkpoint(d, model, opt, CTX, data=data)
    _equal(model.state_dict(), before)


def test_incomplete_and_invalid(tmp_path):
    model, opt, data = _state(tmp_path)
    d = tmp_path / "ck"
    checkpoint.save_checkpoint(d, model, opt, CTX, step=3, data=data)
    (d / "manifest.pt").unlink()
    with pytest.raises(RuntimeError, match="incomplete"):
        checkpoint.load_checkpoint(d, model, opt, CTX, data=data)
    with pytest.raises(ValueError, match="step"):
        checkpoint.save_checkpoint(tmp_path / "x", model, opt, CTX, step=-1, data=data)
