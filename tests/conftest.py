"""Test configuration: markers and import path.

Markers:
  gpu          needs a CUDA device (run on a B200 with ``-m gpu``)
  distributed  spawns local Gloo / torchrun processes (CPU)
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "distributed: launches local Gloo or torchrun processes")
