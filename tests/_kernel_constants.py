"""Constants read from the CUDA sources, so the protocol model checks follow
the kernels when a ring depth changes."""

import os
import re

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "nano_megatron_b200", "csrc")


def constant(filename: str, name: str) -> int:
    with open(os.path.join(CSRC, filename)) as f:
        text = f.read()
    m = re.search(rf"\b{name}\s*=\s*(\d+)\s*[;,]", text)
    if m is None:
        raise LookupError(f"{name} not found in {filename}")
    return int(m.group(1))
