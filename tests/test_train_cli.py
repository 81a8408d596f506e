"""End-to-end ``torchrun`` CLI: two steps straight through must produce
bit-identical rank shards (model, optimizer, RNG, data cursor) to one step,
save, restart from the checkpoint, one more step (TP=2 PP=2 SP recompute
bf16); DP=2 x PP=2 with the gradient bucketer must match one average after
backward bit for bit; a save format the model does not fit is refused at
startup."""

import socket
import struct
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).parents[1]
pytestmark = pytest.mark.distributed


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(out, tokens, steps, load=None, layout=("--tp=2", "--pp=2"), extra=()):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=4",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", "-m", "nano_megatron_b200.train",
           *layout, f"--steps={steps}", "--num-microbatches=2", "--micro-batch-size=1",
           "--n-layer=2", "--n-head=4", "--n-embd=32", "--vocab-size=64", "--seq-len=8",
           "--ffn-hidden-size=48", "--sequence-parallel", "--recompute", "--dtype=bfloat16",
           f"--data={tokens}", f"--save={out}", *extra]
    if load is not None:
        cmd.append(f"--load={load}")
    env = dict(__import__("os").environ, OMP_NUM_THREADS="1")
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=240, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


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


def test_interrupted_training_matches_uninterrupted(tmp_path):
    tokens = tmp_path / "tokens.bin"
    tokens.write_bytes(struct.pack("=4096H", *(i % 64 for i in range(4096))))
    out = _run(tmp_path / "continuous", tokens, 2)
    assert "step   1 | loss" in out
    _run(tmp_path / "split", tokens, 1)
    _run(tmp_path / "resumed", tokens, 2, load=tmp_path / "split" / "step_00000001")
    a, b = tmp_path / "continuous" / "step_00000002", tmp_path / "resumed" / "step_00000002"
    for d in (a, b):
        assert (d / "manifest.pt").is_file() and len(list(d.glob("rank_*.pt"))) == 4
    for r in range(4):
        name = f"rank_{r:05d}.pt"
        _equal(torch.load(b / name, weights_only=False), torch.load(a / name, weights_only=False))


def test_dp_buckets_match_one_average_after_backward(tmp_path):
    """DP=2 x PP=2: gradients averaged bucket by bucket during the last backward
    (tiny buckets, so many) give bit-identical shards to one average after it."""
    tokens = tmp_path / "tokens.bin"
    tokens.write_bytes(struct.pack("=4096H", *(i % 64 for i in range(4096))))
    layout = ("--tp=1", "--pp=2", "--dp=2")
    _run(tmp_path / "buckets", tokens, 2, layout=layout, extra=("--dp-bucket-mb=0.002",))
    _run(tmp_path / "single", tokens, 2, layout=layout, extra=("--dp-bucket-mb=0",))
    a, b = tmp_path / "single" / "step_00000002", tmp_path / "buckets" / "step_00000002"
    for r in range(4):
        name = f"rank_{r:05d}.pt"
        _equal(torch.load(b / name, weights_only=False), torch.load(a / name, weights_only=False))


def test_reference_save_format_is_checked_before_training(tmp_path):
    """A model the reference cannot describe is refused at startup, not at the first save."""
    import os
    env = dict(os.environ, OMP_NUM_THREADS="1", RANK="0", LOCAL_RANK="0", WORLD_SIZE="1",
               MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_port()))
    cmd = [sys.executable, "-m", "nano_megatron_b200.train", "--steps=3", "--ffn-hidden-size=96",
           "--save-format=reference", f"--save={tmp_path / 'out'}"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=120, env=env)
    assert r.returncode != 0 and "SwiGLU width 96" in r.stderr
    assert "step   0" not in r.stdout and not (tmp_path / "out").exists()
