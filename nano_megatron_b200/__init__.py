"""nano_megatron_b200: a Megatron-style TP x SP x PP x DP GPT trainer for NVIDIA B200.

PyTorch is the framework layer; the CUDA hot path is hand-written sm_100a
kernels (``nano_megatron_b200/csrc``) and the CPU path is plain torch math that
serves as the correctness oracle.
"""

from .models import GPT, GPTConfig
from .parallel import ParallelContext, init_parallel
from .parallel.pipeline import forward_backward_1f1b

__all__ = ["GPT", "GPTConfig", "ParallelContext", "init_parallel", "forward_backward_1f1b"]
