"""GPT model family: config, tensor-parallel layers, the stage model."""

from .config import GPTConfig, divide
from .gpt import (GPT, ParallelAttention, ParallelLMHead, ParallelMLP, TransformerLayer,
                  build_rope_cache, layers_for_stage)
from .layers import ColumnParallelLinear, RMSNorm, RowParallelLinear, VocabParallelEmbedding

__all__ = [
    "GPT", "GPTConfig", "divide", "ParallelAttention", "ParallelLMHead", "ParallelMLP",
    "TransformerLayer", "build_rope_cache", "layers_for_stage", "ColumnParallelLinear",
    "RMSNorm", "RowParallelLinear", "VocabParallelEmbedding",
]
