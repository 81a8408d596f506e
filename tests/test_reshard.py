"""Resharding a checkpoint to another layout (``utils/reshard.py``).

A TP=2 x PP=2 run with sequence parallelism trains two steps through the CLI
on Gloo ranks and saves. Resharding that step to TP=1 and back, or through a
TP=2 x DP=2 layout, gives back every shard's parameters and flat AdamW
moments exactly. Resuming the TP=1 copy for two more steps gives the losses
and weights of the original layout resumed for two more steps, to fp32
rounding. A layout the model does not divide over is refused before anything
is written.
"""

import os
import re
import socket
import struct
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from nano_megatron_b200.utils.reshard import reshard

ROOT = Path(__file__).parents[1]
pytestmark = pytest.mark.distributed
MODEL = ["--sequence-parallel", "--num-microbatches=2", "--micro-batch-size=2", "--n-layer=2", "--n-head=4",
         "--n-embd=32", "--vocab-size=64", "--seq-len=8", "--lr=0.001"]


def _train(nproc, flags, tmp_path, tokens):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={port}", "-m", "nano_megatron_b200.train",
           *MODEL, f"--data={tokens}", *flags]
    env = dict(os.environ, OMP_NUM_THREADS="1", PYTHONPATH=str(ROOT))
    r = subprocess.run(cmd, cwd=tmp_path, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    return [float(x) for x in re.findall(r"loss (\d+\.\d+)", r.stdout)]


def _shards(step_dir):
    manifest = torch.load(step_dir / "manifest.pt", weights_only=False)
    return [torch.load(step_dir / name, weights_only=False) for name in manifest["shards"]]


@pytest.fixture(scope="module")
def source(tmp_path_factory):
    tmp = tmp_path_factory.mktemp("reshard")
    tokens = tmp / "tokens.bin"
    tokens.write_bytes(struct.pack("=4096H", *((11 * i + 2) % 64 for i in range(4096))))
    _train(4, ["--tp=2", "--pp=2", "--steps=2", f"--save={tmp / 'run'}"], tmp, tokens)
    return tmp, tokens, tmp / "run" / "step_00000002"


def test_round_trips_are_exact(source):
    tmp, _, step = source
    one = reshard(step, tmp / "tp1", tp=1, pp=1)
    back = reshard(one, tmp / "back", tp=2, pp=2)
    via_dp = reshard(reshard(step, tmp / "tp2dp2", tp=2, pp=1, dp=2), tmp / "back2", tp=2, pp=2)
    original = _shards(step)
    assert len(_shards(one)) == 1 and len(_shards(tmp / "tp2dp2")) == 4
    for copy in (back, via_dp):
        copied = _shards(copy)
        assert len(copied) == len(original) == 4
        for a, b in zip(original, copied):
            assert a["topology"] == b["topology"] and a["step"] == b["step"] and a["extra"] == b["extra"]
            assert a["data"] == b["data"]
            assert a["model"].keys() == b["model"].keys()
            assert all(torch.equal(a["model"][k], b["model"][k]) for k in a["model"])
            sa, sb = a["optimizer"]["state"], b["optimizer"]["state"]
            assert sa["step"] == sb["step"] and a["optimizer"]["param_groups"] == b["optimizer"]["param_groups"]
            assert torch.equal(sa["exp_avg"], sb["exp_avg"]) and torch.equal(sa["exp_avg_sq"], sb["exp_avg_sq"])
    dp_shards = _shards(tmp / "tp2dp2")
    assert [s["data"]["layout"]["dp_rank"] for s in dp_shards] == [0, 0, 1, 1]


def test_resumed_at_another_layout_trains_the_same(source):
    tmp, tokens, step = source
    reshard(step, tmp / "tp1_resume" / "step_00000002", tp=1, pp=1)
    losses_tp1 = _train(1, ["--steps=4", f"--load={tmp / 'tp1_resume' / 'step_00000002'}",
                            f"--save={tmp / 'tp1_resume'}"], tmp, tokens)
    losses_tp2pp2 = _train(4, ["--tp=2", "--pp=2", "--steps=4", f"--load={step}",
                               f"--save={tmp / 'tp2pp2_resume'}"], tmp, tokens)
    assert len(losses_tp1) == len(losses_tp2pp2) == 2
    torch.testing.assert_close(torch.tensor(losses_tp1), torch.tensor(losses_tp2pp2), rtol=1e-4, atol=1e-5)
    gathered = reshard(tmp / "tp2pp2_resume" / "step_00000004", tmp / "gathered", tp=1, pp=1)
    a, b = _shards(tmp / "tp1_resume" / "step_00000004")[0], _shards(gathered)[0]
    for k in a["model"]:
        torch.testing.assert_close(a["model"][k], b["model"][k], rtol=1e-4, atol=1e-6, msg=k)


def test_a_layout_the_model_does_not_divide_over_is_refused(source):
    tmp, _, step = source
    with pytest.raises(ValueError):
        reshard(step, tmp / "tp3", tp=3, pp=1)
    assert not (tmp / "tp3").exists()
    with pytest.raises(ValueError, match="source"):
        reshard(step, step, tp=1, pp=1)
    assert (step / "manifest.pt").exists()


def test_untied_embeddings_round_trip(source, tmp_path):
    _, tokens, _ = source
    _train(4, ["--tp=2", "--pp=2", "--steps=1", "--untie-embeddings", f"--save={tmp_path / 'run'}"],
           tmp_path, tokens)
    step = tmp_path / "run" / "step_00000001"
    back = reshard(reshard(step, tmp_path / "tp1", tp=1, pp=1), tmp_path / "back", tp=2, pp=2)
    one = _shards(tmp_path / "tp1")[0]["model"]
    assert not torch.equal(one["embedding.weight"], one["lm_head.weight"])
    original, copied = _shards(step), _shards(back)
    assert len(original) == len(copied) == 4
    for a, b in zip(original, copied):
        assert a["model"].keys() == b["model"].keys()
        assert all(torch.equal(a["model"][k], b["model"][k]) for k in a["model"])
        assert torch.equal(a["optimizer"]["state"]["exp_avg_sq"], b["optimizer"]["state"]["exp_avg_sq"])


def test_a_manifest_that_disagrees_with_its_shards_is_refused(source, tmp_path):
    import shutil

    from nano_megatron_b200.utils.checkpoint import CheckpointError
    _, _, step = source
    copy = tmp_path / "copy"
    shutil.copytree(step, copy)
    manifest = torch.load(copy / "manifest.pt", weights_only=False)
    manifest["parallel_sizes"] = {"tp": 4, "pp": 1, "dp": 1}
    torch.save(manifest, copy / "manifest.pt")
    with pytest.raises(CheckpointError, match="topology"):
        reshard(copy, tmp_path / "out", tp=1, pp=1)
    assert not (tmp_path / "out").exists()
