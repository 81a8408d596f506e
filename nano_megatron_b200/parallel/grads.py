"""Gradient finalization, initial parameter sync and logical-norm clipping.

After the pipeline backward:

1. TP-replicated parameters (RMSNorm weights, replicated biases) are summed
   over the TP group: averaged without sequence parallelism (every TP rank saw
   the same tokens), kept as a SUM with it (ranks saw disjoint tokens). All
   replicated gradients travel in ONE coalesced all-reduce.
2. Tied embedding copies on the first and last pipeline stages are summed over
   the tied group.
3. Data-parallel replicas average their gradients. On a model with flat
   buffers this is one all-reduce of the flat gradient buffer (or, with a
   :class:`GradBucketer`, bucket by bucket overlapped with the last backward).

Clipping uses the L2 norm of the logical unsharded model accumulated in
fp64: TP shards add, replicated parameters count ``1/tp``, pipeline stages add,
DP is never reduced, and a tied last-stage LM head is counted once.

Parity: ``nano_megatron/grads.py:16-193``.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .context import ParallelContext


def _is_sharded(param) -> bool:
    return getattr(param, "tensor_parallel_sharded", False)


def _flat_buffers(model):
    return getattr(model, "flat_buffers", None)


def all_reduce_replicated_gradients(model, ctx: ParallelContext, *, sequence_parallel: bool = False) -> None:
    """One coalesced all-reduce of every TP-replicated gradient (the reference
    reduces each one on its own, ``nano_megatron/grads.py:16-32``): a SUM with
    sequence parallelism, the TP mean without."""
    if ctx.tp_size == 1:
        return
    grads = [p.grad for p in model.parameters() if p.grad is not None and not _is_sharded(p)]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, group=ctx.tp_group)
    if not sequence_parallel:
        flat /= ctx.tp_size
    offset = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[offset: offset + n].view_as(g))
        offset += n


def all_reduce_data_parallel_gradients(model, ctx: ParallelContext) -> None:
    """Average gradients over the DP group (flat buffer: one collective).
    Parity: ``nano_megatron/grads.py:35-54``."""
    if ctx.dp_size == 1:
        return
    buffers = _flat_buffers(model)
    if buffers is not None:
        _dp_average(buffers.grad, ctx)
        return
    by_key: dict = {}
    for p in model.parameters():
        if p.grad is not None:
            by_key.setdefault((p.grad.device, p.grad.dtype), []).append(p.grad)
    for grads in by_key.values():
        flat = torch.cat([g.reshape(-1) for g in grads])
        _dp_average(flat, ctx)
        offset = 0
        for g in grads:
            n = g.numel()
            g.copy_(flat[offset: offset + n].view_as(g))
            offset += n


def _dp_average(flat: torch.Tensor, ctx: ParallelContext) -> None:
    if flat.is_cuda:
        # NCCL folds the 1/dp scale into the reduction (pre-multiplied sum).
        dist.all_reduce(flat, op=dist.ReduceOp.AVG, group=ctx.dp_group)
    else:
        dist.all_reduce(flat, group=ctx.dp_group)
        flat /= ctx.dp_size


class GradBucketer:
    """Data-parallel gradient averaging in buckets, started during the last backward.

    The stage's flat gradient buffer is cut into buckets of whole regions,
    about ``bucket_bytes`` each, formed from the end of the buffer (the last
    layers, whose gradients backward produces first). Every kernel that
    accumulates into a region reports it (``functional.set_grad_observer``);
    the backwards before the last one teach the bucketer how many writes a
    region receives per microbatch (two for an embedding tied to the LM head
    on one stage), and during the final microbatch's backward a region is
    complete once it received that many. When every region of a bucket is
    complete, the bucket's reduction starts: on CUDA on a communication
    stream that first waits for an event recorded after the last write. The
    reduction is ``reducer(start, end)`` when given -- on CUDA the NVLink
    kernel of :mod:`nano_megatron_b200.ops.dp_reduce`, which applies the
    ``1/dp`` scale in the same pass -- else NCCL ``ReduceOp.AVG``.
    :meth:`finish` starts whatever is left (a step with one microbatch learns
    nothing the first time and reduces everything there) and makes the compute
    stream wait for all of it.

    ``overlap=False`` issues each bucket on the compute stream instead (still
    bucket by bucket, still started during backward). ``last_step`` records,
    after :meth:`finish`, how many buckets started during the last backward
    and how many only in :meth:`finish`.

    Parity: replaces ``nano_megatron/grads.py:35-54`` (one flat all-reduce
    after the whole backward, then a division by ``dp``).
    """

    def __init__(self, model, ctx: ParallelContext, bucket_bytes: int = 128 << 20, overlap: bool = True,
                 reducer=None):
        buffers = _flat_buffers(model)
        if buffers is None:
            raise ValueError("the bucketer needs a model with flat gradient buffers")
        self.ctx = ctx
        self.grad = buffers.grad
        regions = buffers.regions
        self.region_of_ptr: dict[int, int] = {}
        for i, region in enumerate(regions):
            self.region_of_ptr[region.grad_block.data_ptr()] = i
            for p in region.params:
                self.region_of_ptr[p.main_grad.data_ptr()] = i
        # buckets of consecutive regions, from the end of the buffer
        limit = max(1, bucket_bytes // self.grad.element_size())
        self.buckets: list[tuple[int, int]] = []       # [start, end) element spans
        self.bucket_regions: list[list[int]] = []
        self.bucket_of = [0] * len(regions)
        end = buffers.numel
        current: list[int] = []
        for i in range(len(regions) - 1, -1, -1):
            current.append(i)
            start = regions[i].offset
            if end - start >= limit or i == 0:
                b = len(self.buckets)
                self.buckets.append((0 if i == 0 else start, end))
                self.bucket_regions.append(current)
                for r in current:
                    self.bucket_of[r] = b
                end, current = start, []
        # ``reducer(start, end)`` averages one span in place on the current
        # stream (our NVLink kernel); None means NCCL all_reduce(AVG).
        self.reducer = reducer
        self.overlap = overlap and self.grad.is_cuda
        self.stream = torch.cuda.Stream(device=self.grad.device) if self.overlap else None
        self.per_microbatch: list[int] | None = None
        self.last_step = {"during_backward": 0, "in_finish": 0, "on_comm_stream": self.overlap}
        self._reset()

    def _reset(self) -> None:
        self.writes = [0] * len(self.bucket_of)
        self.armed = False
        self.left: list[int] = []
        self.bucket_left: list[int] = []
        self.started = [False] * len(self.buckets)
        self.works: list = []

    # ------------------------------------------------------------ observers
    def observe(self, tensor) -> None:
        i = self.region_of_ptr.get(tensor.data_ptr())
        if i is None:
            return
        self.writes[i] += 1
        if self.armed and self.left[i] > 0:
            self.left[i] -= 1
            if self.left[i] == 0:
                b = self.bucket_of[i]
                self.bucket_left[b] -= 1
                if self.bucket_left[b] == 0:
                    self._start(b)

    def before_last_backward(self, prior_backwards: int) -> None:
        if prior_backwards > 0:
            self.per_microbatch = [w // prior_backwards for w in self.writes]
        if self.per_microbatch is None:
            return
        self.left = list(self.per_microbatch)
        self.bucket_left = [sum(1 for r in regions if self.left[r] > 0) for regions in self.bucket_regions]
        self.armed = True
        for b, n in enumerate(self.bucket_left):
            if n == 0:
                self._start(b)

    # ----------------------------------------------------------- reduction
    def _start(self, b: int) -> None:
        if self.started[b]:
            return
        self.started[b] = True
        start, end = self.buckets[b]
        view = self.grad[start:end]
        if self.reducer is not None and self.stream is not None:
            ready = torch.cuda.Event()
            ready.record(torch.cuda.current_stream(self.grad.device))
            self.stream.wait_event(ready)
            with torch.cuda.stream(self.stream):
                self.reducer(start, end)
        elif self.reducer is not None:
            self.reducer(start, end)
        elif self.stream is not None:
            ready = torch.cuda.Event()
            ready.record(torch.cuda.current_stream(self.grad.device))
            self.stream.wait_event(ready)
            with torch.cuda.stream(self.stream):
                self.works.append(dist.all_reduce(view, op=dist.ReduceOp.AVG, group=self.ctx.dp_group,
                                                  async_op=True))
        elif view.is_cuda:
            dist.all_reduce(view, op=dist.ReduceOp.AVG, group=self.ctx.dp_group)
        else:
            self.works.append((dist.all_reduce(view, group=self.ctx.dp_group, async_op=True), view))

    def finish(self) -> None:
        """Start the remaining buckets (in bucket order) and wait for every bucket."""
        early = sum(self.started)
        self.last_step = {"during_backward": early, "in_finish": len(self.buckets) - early,
                          "on_comm_stream": self.overlap}
        for b in range(len(self.buckets)):
            self._start(b)
        for work in self.works:
            if isinstance(work, tuple):
                work[0].wait()
                work[1].div_(self.ctx.dp_size)
            else:
                work.wait()
        if self.stream is not None:
            torch.cuda.current_stream(self.grad.device).wait_stream(self.stream)
        self._reset()


def all_reduce_embedding_gradients(model, ctx: ParallelContext) -> None:
    """SUM the tied embedding / LM-head gradient copies over the tied group.
    Parity: ``nano_megatron/grads.py:57-78``."""
    if ctx.pp_size == 1 or ctx.tied_group is None:
        return
    if not (ctx.is_first_stage or ctx.is_last_stage):
        return
    module = getattr(model, "embedding" if ctx.is_first_stage else "lm_head", None)
    if module is None or module.weight.grad is None:
        return
    dist.all_reduce(module.weight.grad, group=ctx.tied_group)


def synchronize_tied_embeddings(model, ctx: ParallelContext) -> None:
    """Broadcast the first stage's embedding into the last stage's LM head.
    Parity: ``nano_megatron/grads.py:81-102``."""
    if ctx.pp_size == 1 or ctx.tied_group is None:
        return
    if not (ctx.is_first_stage or ctx.is_last_stage):
        return
    module = getattr(model, "embedding" if ctx.is_first_stage else "lm_head", None)
    if module is None:
        return
    dist.broadcast(module.weight.data, src=ctx.pp_ranks[0], group=ctx.tied_group)


def synchronize_model_parameters(model, ctx: ParallelContext, *, tie_embeddings: bool = False) -> None:
    """Make replicated parameters agree after rank-dependent initialization.
    Parity: ``nano_megatron/grads.py:105-127``."""
    if ctx.tp_size > 1:
        for p in model.parameters():
            if not _is_sharded(p):
                dist.broadcast(p.data, src=ctx.tp_ranks[0], group=ctx.tp_group)
    if ctx.dp_size > 1:
        buffers = _flat_buffers(model)
        if buffers is not None:
            dist.broadcast(buffers.data, src=ctx.dp_ranks[0], group=ctx.dp_group)
        else:
            for p in model.parameters():
                dist.broadcast(p.data, src=ctx.dp_ranks[0], group=ctx.dp_group)
    if tie_embeddings:
        synchronize_tied_embeddings(model, ctx)
    refresh = getattr(model, "refresh_compute_copies", None)
    if refresh is not None:
        refresh()


def finalize_gradients(model, ctx: ParallelContext, *, tie_embeddings: bool = False,
                       sequence_parallel: bool = False, skip_data_parallel: bool = False) -> None:
    """Replicated-TP, then tied, then DP reduction (``skip_data_parallel`` when a
    bucketer already reduced the DP gradients during backward).
    Parity: ``nano_megatron/grads.py:130-140``."""
    all_reduce_replicated_gradients(model, ctx, sequence_parallel=sequence_parallel)
    if tie_embeddings:
        all_reduce_embedding_gradients(model, ctx)
    if not skip_data_parallel:
        all_reduce_data_parallel_gradients(model, ctx)


def _norm_terms(model, ctx: ParallelContext, tie_embeddings: bool):
    """``(param, weight)`` pairs: each grad's squared norm counts ``weight`` times."""
    terms = []
    for name, p in model.named_parameters():
        if p.grad is None:
            continue
        if tie_embeddings and ctx.pp_size > 1 and ctx.is_last_stage and name == "lm_head.weight":
            continue  # the same logical parameter as the first stage's embedding
        terms.append((p, 1.0 if _is_sharded(p) else 1.0 / ctx.tp_size))
    return terms


def grad_norm_squared(model, ctx: ParallelContext, *, tie_embeddings: bool = False) -> torch.Tensor:
    """Logical-model squared gradient norm (fp64), reduced over TP then PP
    and never over DP (``nano_megatron/grads.py:162-187``)."""
    params = list(model.parameters())
    device = params[0].device if params else torch.device("cpu")
    terms = _norm_terms(model, ctx, tie_embeddings)
    buffers = _flat_buffers(model)
    if device.type == "cuda" and terms and buffers is not None:
        # One pass over the flat gradient buffer, region by region (a fused
        # q|k|v or gate|up region holds parameters with one common weight).
        from .. import ops
        weight_of = {id(p): w for p, w in terms}
        blocks, weights = [], []
        for region in buffers.regions:
            w = weight_of.get(id(region.params[0]))
            if w is not None:
                blocks.append(region.grad_block)
                weights.append(w)
        total = ops.cuda_ops().weighted_sq_norm(blocks, weights)
    else:
        total = torch.zeros((), dtype=torch.float64, device=device)
        for p, w in terms:
            total += p.grad.detach().double().pow(2).sum() * w
    if ctx.tp_size > 1:
        dist.all_reduce(total, group=ctx.tp_group)
    if ctx.pp_size > 1:
        dist.all_reduce(total, group=ctx.pp_group)
    return total


def clip_coefficient(total_norm: torch.Tensor, max_norm: float) -> torch.Tensor:
    """``min(1, max_norm / (norm + 1e-6))`` as a device tensor."""
    return torch.clamp(max_norm / (total_norm + 1e-6), max=1.0)


def clip_grad_norm(model, ctx: ParallelContext, max_norm: float, *, tie_embeddings: bool = False,
                   apply: bool = True) -> torch.Tensor:
    """Clip every gradient by the logical-model norm; return that norm (fp64).

    With ``apply=False`` the gradients are left untouched and the caller
    applies the coefficient itself (the fused optimizer does it on load).
    Parity: ``nano_megatron/grads.py:143-193``.
    """
    if max_norm < 0:
        raise ValueError(f"max_norm must be non-negative, got {max_norm}")
    total_norm = grad_norm_squared(model, ctx, tie_embeddings=tie_embeddings).sqrt()
    if apply:
        coefficient = clip_coefficient(total_norm, max_norm)
        buffers = _flat_buffers(model)
        if buffers is not None:
            buffers.grad.mul_(coefficient.to(buffers.grad.dtype))
        else:
            for p in model.parameters():
                if p.grad is not None:
                    p.grad.mul_(coefficient.to(dtype=p.grad.dtype))
    return total_norm
