"""Real Gloo processes: sequence all-gather / reduce-scatter values and their
adjoint gradients, sequence-first (dim 0) and batch-first (dim 1, the default
of the public functions, as in the reference)."""

import os
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nano_megatron_b200.parallel import (gather_from_sequence_parallel_region, init_parallel,
                                         reduce_scatter_to_sequence_parallel_region)

pytestmark = pytest.mark.distributed


def _worker(rank, world, init_file, q):
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        ctx = init_parallel(tp_size=world)
        for dim in (0, 1):
            full = torch.arange(2 * 4 * 3 * 2, dtype=torch.float32).view(4, 2, 3, 2)
            if dim == 1:
                full = full.transpose(0, 1).contiguous()  # [2, 4, 3, 2]
            shard = torch.chunk(full, world, dim=dim)[rank].clone().requires_grad_(True)
            kw = {"seq_dim": 0} if dim == 0 else {}
            gathered = gather_from_sequence_parallel_region(shard, ctx, **kw)
            torch.testing.assert_close(gathered, full)
            gathered.square().sum().backward()
            torch.testing.assert_close(shard.grad, torch.chunk(2 * full, world, dim=dim)[rank] * world)
            partial = (full / world).requires_grad_(True)
            reduced = reduce_scatter_to_sequence_parallel_region(partial, ctx, **kw)
            torch.testing.assert_close(reduced, torch.chunk(full, world, dim=dim)[rank])
            reduced.sum().backward()
            torch.testing.assert_close(partial.grad, torch.ones_like(full))
        q.put(rank)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sequence_collectives(world):
    mpctx = mp.get_context("spawn")
    q = mpctx.Queue()
    with tempfile.TemporaryDirectory() as tmp:
        init = os.path.join(tmp, "rdv")
        procs = [mpctx.Process(target=_worker, args=(r, world, init, q)) for r in range(world)]
        for p in procs:
            p.start()
        got = sorted(q.get(timeout=60) for _ in procs)
        for p in procs:
            p.join(timeout=60)
    assert got == list(range(world))
    assert all(p.exitcode == 0 for p in procs)
