"""Moving a run from the reference's command line to this package's, through
``torchrun`` on Gloo ranks (the reference is installed under ``baseline/_ref``
or the directory named by ``NMB_REFERENCE_PATH``; skipped when neither holds
the ``nano_megatron`` package).

The reference CLI trains four steps at TP=2, and at TP=2 x PP=2, with sequence
parallelism on a token file, saving at step 2 and step 4. This package's CLI resumes the step-2
directory with ``--load-reference`` and trains to step 4. Every rank's model
state and data cursor at step 4 must match the reference's uninterrupted run.
The other direction: this package's CLI saves in the reference's format
(``--save-format reference``) and the reference's CLI resumes that step-2
directory with its own ``--load``.
"""

import os
import socket
import struct
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).parents[1]
REF = os.environ.get("NMB_REFERENCE_PATH") or str(ROOT / "baseline" / "_ref")
pytestmark = pytest.mark.distributed

COMMON = ["--sequence-parallel", "--num-microbatches=2", "--micro-batch-size=2", "--n-layer=2",
          "--n-head=4", "--n-embd=32", "--vocab-size=64", "--seq-len=8", "--lr=0.001"]
LAYOUTS = {"tp2-sp": (["--tp=2"], 2), "tp2xpp2-sp": (["--tp=2", "--pp=2"], 4), "dp2": (["--dp=2"], 2)}


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _torchrun(module, args, pythonpath, nproc):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", "-m", module, *args]
    env = dict(os.environ, OMP_NUM_THREADS="1", PYTHONPATH=pythonpath)
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.parametrize("layout", sorted(LAYOUTS))
def test_reference_run_continues_in_this_package(tmp_path, layout):
    if not os.path.isdir(os.path.join(REF, "nano_megatron")):
        pytest.skip(f"reference package not found under {REF}")
    flags, nproc = LAYOUTS[layout]
    tokens = tmp_path / "tokens.bin"
    tokens.write_bytes(struct.pack("=4096H", *((7 * i + 3) % 64 for i in range(4096))))
    ref_out, our_out = tmp_path / "reference", tmp_path / "ours"
    _torchrun("nano_megatron.train", flags + COMMON + ["--steps=4", "--save-every=2", f"--data={tokens}",
                                                       f"--save={ref_out}"], REF, nproc)
    _torchrun("nano_megatron_b200.train", flags + COMMON + ["--steps=4", f"--data={tokens}", f"--save={our_out}",
                                                            f"--load-reference={ref_out / 'step_00000002'}"],
              str(ROOT), nproc)
    a, b = ref_out / "step_00000004", our_out / "step_00000004"
    for rank in range(nproc):
        ref_shard = torch.load(a / f"rank_{rank:05d}.pt", weights_only=False)
        our_shard = torch.load(b / f"rank_{rank:05d}.pt", weights_only=False)
        assert our_shard["step"] == ref_shard["step"] == 4
        assert our_shard["data"]["cursor"] == ref_shard["data"]["cursor"]
        assert our_shard["model"].keys() == ref_shard["model"].keys()
        for name, value in ref_shard["model"].items():
            torch.testing.assert_close(our_shard["model"][name], value, rtol=1e-4, atol=1e-6, msg=name)


@pytest.mark.parametrize("layout", sorted(LAYOUTS))
def test_this_package_run_continues_in_the_reference(tmp_path, layout):
    if not os.path.isdir(os.path.join(REF, "nano_megatron")):
        pytest.skip(f"reference package not found under {REF}")
    flags, nproc = LAYOUTS[layout]
    tokens = tmp_path / "tokens.bin"
    tokens.write_bytes(struct.pack("=4096H", *((5 * i + 1) % 64 for i in range(4096))))
    our_out, ref_out = tmp_path / "ours", tmp_path / "reference"
    _torchrun("nano_megatron_b200.train", flags + COMMON + ["--steps=4", "--save-every=2", "--save-format=reference",
                                                            f"--data={tokens}", f"--save={our_out}"], str(ROOT), nproc)
    _torchrun("nano_megatron.train", flags + COMMON + ["--steps=4", f"--data={tokens}", f"--save={ref_out}",
                                                       f"--load={our_out / 'step_00000002'}"], REF, nproc)
    a, b = our_out / "step_00000004", ref_out / "step_00000004"
    for rank in range(nproc):
        our_shard = torch.load(a / f"rank_{rank:05d}.pt", weights_only=False)
        ref_shard = torch.load(b / f"rank_{rank:05d}.pt", weights_only=False)
        assert our_shard["step"] == ref_shard["step"] == 4
        assert our_shard["data"]["cursor"] == ref_shard["data"]["cursor"]
        assert our_shard["model"].keys() == ref_shard["model"].keys()
        for name, value in our_shard["model"].items():
            torch.testing.assert_close(ref_shard["model"][name], value, rtol=1e-4, atol=1e-6, msg=name)
