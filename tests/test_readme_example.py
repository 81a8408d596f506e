"""The Python example in README.md runs as written (on one CPU process, in a
scratch directory, on a free local port)."""

import os
import re
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).parents[1]
pytestmark = pytest.mark.distributed


def test_readme_python_example_runs(tmp_path):
    blocks = re.findall(r"```python\n(.*?)```", (ROOT / "README.md").read_text(), re.S)
    assert blocks, "README.md has no python example"
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    code = re.sub(r"tcp://127\.0\.0\.1:\d+", f"tcp://127.0.0.1:{port}", blocks[0])
    env = dict(os.environ, PYTHONPATH=str(ROOT), OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, "-c", code], cwd=tmp_path, env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.split("\n")
    assert [ln.split()[0] for ln in lines if ln.strip()] == ["0", "1", "2"]
    assert (tmp_path / "ckpt" / "step_00000003" / "manifest.pt").exists()
