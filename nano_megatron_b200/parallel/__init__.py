"""Process grid, TP/SP collectives, pipeline schedule and gradient finalization."""

from .context import ParallelContext, init_parallel
from .mappings import (copy_to_tensor_parallel_region, gather_from_sequence_parallel_region,
                       reduce_from_tensor_parallel_region,
                       reduce_scatter_to_sequence_parallel_region)

__all__ = [
    "ParallelContext", "init_parallel", "copy_to_tensor_parallel_region",
    "gather_from_sequence_parallel_region", "reduce_from_tensor_parallel_region",
    "reduce_scatter_to_sequence_parallel_region",
]
