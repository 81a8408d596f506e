"""Checkpoints: a resumed run continues bit for bit; a save that fails half way
(fault injected on the host) leaves no partial file and no manifest; damaged
manifests and shards (truncated, corrupted, wrong step) are refused before any
state changes; every mismatch is reported in one error."""

import copy
from dataclasses import replace
from unittest import mock

import numpy as np
import pytest
import torch

from nano_megatron_b200.models import GPT, GPTConfig
from nano_megatron_b200.optim import FusedAdamW
from nano_megatron_b200.parallel import ParallelContext
from nano_megatron_b200.utils import checkpoint as ck
from nano_megatron_b200.utils.data import TokenStream

SOLO = ParallelContext.single()
CFG = GPTConfig(vocab_size=96, n_layer=2, n_head=4, n_embd=32, seq_len=6, ffn_hidden_size=48)


def _run(seed, tmp_path):
    torch.manual_seed(seed)
    model = GPT(CFG)
    path = tmp_path / "ids.bin"
    if not path.exists():
        np.arange(5000, dtype="=u2").__imod__(96).tofile(path)
    return model, FusedAdamW(model, lr=3e-3), TokenStream(path, dtype="uint16", seq_len=6)


def _train(model, opt, stream, steps):
    losses = []
    for _ in range(steps):
        opt.zero_grad()
        x, y = stream.next_batch(3)
        loss = model(x, y)
        loss.backward()
        opt.step()
        losses.append(loss.item())
    return losses


def _snapshot(model):
    return {k: v.clone() for k, v in model.state_dict().items()}


def _unchanged(model, snap):
    return all(torch.equal(v, snap[k]) for k, v in model.state_dict().items())


def test_resumed_run_continues_bit_for_bit(tmp_path):
    model, opt, stream = _run(5, tmp_path)
    _train(model, opt, stream, 2)
    ck.save_checkpoint(tmp_path / "s2", model, opt, SOLO, step=2, data=stream, extra={"lr": 3e-3})
    noise_after_save = torch.rand(3)
    expected = _train(model, opt, stream, 3)

    other, other_opt, other_stream = _run(99, tmp_path)
    torch.manual_seed(1234)
    step, extra = ck.load_checkpoint(tmp_path / "s2", other, other_opt, SOLO, data=other_stream)
    assert (step, extra) == (2, {"lr": 3e-3})
    assert torch.equal(torch.rand(3), noise_after_save)  # generator states restored
    assert _train(other, other_opt, other_stream, 3) == expected
    base = other.flat_buffers.data  # parameters still view the flat master buffer
    assert all(base.data_ptr() <= p.data_ptr() < base.data_ptr() + 4 * base.numel()
               for p in other.parameters())


def test_failed_save_leaves_no_partial_file_and_no_manifest(tmp_path):
    model, opt, stream = _run(1, tmp_path)
    _train(model, opt, stream, 1)
    ck.save_checkpoint(tmp_path / "s1", model, opt, SOLO, step=1, data=stream)
    target = tmp_path / "s2"
    ck.save_checkpoint(target, model, opt, SOLO, step=2, data=stream)
    before = (target / "rank_00000.pt").read_bytes()

    real_write, calls = ck._Checksummed.write, []

    def dies_midway(self, data):
        calls.append(1)
        if len(calls) == 4:
            raise OSError(28, "No space left on device")
        return real_write(self, data)

    with mock.patch.object(ck._Checksummed, "write", dies_midway):
        with pytest.raises(OSError, match="No space"):
            ck.save_checkpoint(target, model, opt, SOLO, step=3, data=stream)
    assert sorted(p.name for p in target.iterdir()) == ["rank_00000.pt"]
    assert (target / "rank_00000.pt").read_bytes() == before
    with pytest.raises(ck.CheckpointError, match="did not complete"):
        ck.load_checkpoint(target, model, opt, SOLO, data=stream)
    assert ck.load_checkpoint(tmp_path / "s1", model, opt, SOLO, data=stream)[0] == 1


def _damage_truncate_shard(d):
    p = d / "rank_00000.pt"
    p.write_bytes(p.read_bytes()[:-100])


def _damage_flip_shard_byte(d):
    p = d / "rank_00000.pt"
    blob = bytearray(p.read_bytes())
    blob[len(blob) // 2] ^= 0x5A
    p.write_bytes(bytes(blob))


def _damage_truncate_manifest(d):
    p = d / "manifest.pt"
    p.write_bytes(p.read_bytes()[:40])


def _damage_manifest_step(d):
    m = torch.load(d / "manifest.pt", weights_only=False)
    m["step"] = 8
    torch.save(m, d / "manifest.pt")


def _damage_missing_shard_in_list(d):
    m = torch.load(d / "manifest.pt", weights_only=False)
    m["shards"].append("rank_00001.pt")
    torch.save(m, d / "manifest.pt")


@pytest.mark.parametrize("damage, message", [
    (_damage_truncate_shard, "truncated"),
    (_damage_flip_shard_byte, "CRC-32"),
    (_damage_truncate_manifest, "not a readable torch file"),
    (_damage_manifest_step, "step"),
    (_damage_missing_shard_in_list, "missing on disk"),
])
def test_damaged_checkpoint_is_refused_before_any_change(tmp_path, damage, message):
    model, opt, stream = _run(2, tmp_path)
    _train(model, opt, stream, 1)
    d = tmp_path / "s1"
    ck.save_checkpoint(d, model, opt, SOLO, step=7, data=stream)
    damage(d)
    _train(model, opt, stream, 1)
    snap, opt_snap, cursor = _snapshot(model), copy.deepcopy(opt.state_dict()), stream.cursor
    with pytest.raises(ck.CheckpointError, match=message):
        ck.load_checkpoint(d, model, opt, SOLO, data=stream)
    assert _unchanged(model, snap) and stream.cursor == cursor
    assert opt.step_count == opt_snap["state"]["step"]


def test_all_mismatches_are_listed_together(tmp_path):
    model, opt, stream = _run(3, tmp_path)
    ck.save_checkpoint(tmp_path / "s", model, opt, SOLO, step=0, data=stream)
    wider = replace(SOLO, world_size=4, tp_size=2, pp_size=2)
    with pytest.raises(ck.CheckpointError) as err:
        ck.load_checkpoint(tmp_path / "s", model, opt, wider, data=stream)
    text = str(err.value)
    assert "world size: checkpoint 1, this run 4" in text and "parallel sizes" in text

    torch.manual_seed(0)
    bigger = GPT(replace(CFG, n_layer=4))
    with pytest.raises(ck.CheckpointError) as err:
        ck.load_checkpoint(tmp_path / "s", bigger, FusedAdamW(bigger), SOLO)
    text = str(err.value)
    assert "model configuration" in text and "no stream was passed" in text


def test_step_must_be_a_non_negative_int(tmp_path):
    model, opt, _ = _run(4, tmp_path)
    for bad in (-1, 1.0, True):
        with pytest.raises(ValueError, match="step"):
            ck.save_checkpoint(tmp_path / "x", model, opt, SOLO, step=bad)


def test_a_save_root_is_answered_with_its_latest_step(tmp_path):
    model, opt, stream = _run(5, tmp_path)
    root = tmp_path / "ckpt"
    for step in (1, 2):
        _train(model, opt, stream, 1)
        ck.save_checkpoint(root / f"step_{step:08d}", model, opt, SOLO, step=step, data=stream)
    (root / "step_00000003").mkdir()  # an incomplete step (no manifest) is not suggested
    with pytest.raises(ck.CheckpointError, match="step_00000002"):
        ck.load_checkpoint(root, model, opt, SOLO, data=stream)
    with pytest.raises(ck.CheckpointError, match="the save did not complete"):
        ck.load_checkpoint(root / "step_00000003", model, opt, SOLO, data=stream)
