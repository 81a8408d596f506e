"""GPT model family: config, tensor-parallel layers, the stage model."""

from .config import GPTConfig, divide
from .cross_entropy import vocab_parallel_cross_entropy
from .gpt import (GPT, ParallelAttention, ParallelLMHead, ParallelMLP, TransformerLayer, apply_rope,
                  build_rope_cache, cuda_shape_problems, layers_for_stage)
from .layers import ColumnParallelLinear, RMSNorm, RowParallelLinear, VocabParallelEmbedding

__all__ = [
    "GPT", "GPTConfig", "divide", "ParallelAttention", "ParallelLMHead", "ParallelMLP",
    "TransformerLayer", "apply_rope", "build_rope_cache", "layers_for_stage", "ColumnParallelLinear",
    "RMSNorm", "RowParallelLinear", "VocabParallelEmbedding", "vocab_parallel_cross_entropy", "cuda_shape_problems",
]
