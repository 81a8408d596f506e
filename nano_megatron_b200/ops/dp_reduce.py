"""Data-parallel gradient averaging by our own kernel over NVLink peer memory.

The stage's flat fp32 gradient buffer is re-homed into symmetric memory that
every rank of the DP group maps (``torch.distributed._symmetric_memory`` is
used only to allocate and exchange the mappings), next to a small flag area.
``all_reduce_avg(start, end)`` then runs ``csrc/dp_reduce.cu`` on that span:
a two-shot all-reduce (each rank sums its slice over all ranks with peer loads
and writes the average back to every rank with peer stores) with the ``1/dp``
scale in the same pass and bounded flag waits.

Parity: replaces the NCCL average of ``nano_megatron/grads.py:35-54``.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..parallel.context import ParallelContext
from . import cuda as K

TIMEOUT_S = 60.0


class DPWorkspace:
    """Symmetric gradient buffer + flags of one DP group."""

    def __init__(self, ctx: ParallelContext, flat):
        import torch.distributed._symmetric_memory as symm
        self.ctx = ctx
        device = flat.grad.device
        grad = symm.empty(flat.numel, dtype=torch.float32, device=device)
        self.grad_handle = symm.rendezvous(grad, ctx.dp_group)
        flags = symm.empty(K.C.dp_flag_bytes() // 4, dtype=torch.int32, device=device)
        flags.zero_()
        self.flag_handle = symm.rendezvous(flags, ctx.dp_group)
        flat.rehome_grad(grad)
        self.grad, self.flags = grad, flags
        self.grad_ptrs = [int(p) for p in self.grad_handle.buffer_ptrs]
        self.flag_ptrs = [int(p) for p in self.flag_handle.buffer_ptrs]
        self.epoch = 0
        torch.cuda.synchronize(device)
        dist.barrier(group=ctx.dp_group)

    def all_reduce_avg(self, start: int, end: int) -> None:
        """Average ``grad[start:end]`` over the DP group on the current stream."""
        self.epoch += 1
        K.C.dp_allreduce(self.grad_ptrs, self.flag_ptrs, self.ctx.dp_rank, start, end - start, self.epoch,
                         K.status_word(self.grad.device), TIMEOUT_S)
        K._count()
