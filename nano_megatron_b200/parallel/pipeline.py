"""Non-interleaved 1F1B pipeline schedule with point-to-point activation exchange.

Every rank runs the same single-threaded loop. Stage ``r`` of ``p`` first runs
``min(p - r - 1, M)`` warm-up forwards, then alternates one forward and one
backward, then drains the warm-up activations in cool-down backwards. With one
stage the loop is plain gradient accumulation.

Exchanges go through ``torch.distributed.batch_isend_irecv``. In the steady
state a stage pairs its forward send with the receive of the matching output
gradient, and its backward send with the receive of the next activation, so
the two directions of a stage boundary travel in one batched exchange and both
sides always post matching pairs (deadlock-free by construction). On NCCL the
receives are waited on by the compute stream only (no host blocking) and sends
are not waited on at all until the end of the step: the compute stream runs on
while the NCCL stream carries the activation to the next stage.
Activations cross stages batch-first as ``[b, s, H]`` (``s = S/tp`` under
sequence parallelism), the reference's exchange shape.

Parity: ``nano_megatron/pipeline.py:22-224`` (schedule, warm-up depth, P2P
order, loss scaling by ``1/M``).
"""

from __future__ import annotations

import contextlib
import os
from collections.abc import Sequence

import torch
import torch.distributed as dist
import torch.nn as nn

from .context import ParallelContext

Batch = tuple[torch.Tensor, torch.Tensor]


class _P2P:
    """Posts exchanges with the neighbouring stages; defers send completion.
    Parity: ``nano_megatron/pipeline.py:22-108`` (same P2P op order; the
    reference waits on every request at once)."""

    def __init__(self, ctx: ParallelContext, shape, dtype, device):
        self.ctx, self.shape, self.dtype, self.device = ctx, shape, dtype, device
        self.pending_sends: list = []

    def exchange(self, *, send_prev=None, send_next=None, recv_prev=False, recv_next=False):
        ctx = self.ctx
        got_prev = (torch.empty(self.shape, dtype=self.dtype, device=self.device,
                                requires_grad=True) if recv_prev else None)
        got_next = (torch.empty(self.shape, dtype=self.dtype, device=self.device)
                    if recv_next else None)
        ops, send_idx = [], []
        if got_prev is not None:
            ops.append(dist.P2POp(dist.irecv, got_prev, ctx.previous_pipeline_rank))
        if send_next is not None:
            send_idx.append(len(ops))
            ops.append(dist.P2POp(dist.isend, send_next.detach().contiguous(), ctx.next_pipeline_rank))
        if got_next is not None:
            ops.append(dist.P2POp(dist.irecv, got_next, ctx.next_pipeline_rank))
        if send_prev is not None:
            send_idx.append(len(ops))
            ops.append(dist.P2POp(dist.isend, send_prev.detach().contiguous(),
                                  ctx.previous_pipeline_rank))
        if not ops:
            return got_prev, got_next
        works = dist.batch_isend_irecv(ops)
        only_sends = got_prev is None and got_next is None
        for i, work in enumerate(works):
            deferred = (i in send_idx) and (only_sends or self.device.type == "cuda")
            if deferred:
                self.pending_sends.append((work, ops[i].tensor))
            else:
                work.wait()
        return got_prev, got_next

    def drain(self) -> None:
        for work, _ in self.pending_sends:
            work.wait()
        self.pending_sends.clear()


# NVTX ranges around every microbatch forward / backward (for nsys or ncu
# range filters) when NMB_NVTX=1; free otherwise.
_NVTX = os.environ.get("NMB_NVTX", "0") == "1"


def _nvtx(name: str):
    if _NVTX and torch.cuda.is_available():
        return torch.cuda.nvtx.range(name)
    return contextlib.nullcontext()


def _forward_step(model, batch, hidden, losses, num_microbatches, ctx):
    with _nvtx(f"forward stage {ctx.pp_rank}"):
        return _forward_step_impl(model, batch, hidden, losses, num_microbatches, ctx)


def _forward_step_impl(model, batch, hidden, losses, num_microbatches, ctx):
    inputs, labels = batch
    stage_input = inputs if ctx.is_first_stage else hidden
    if stage_input is None:
        raise RuntimeError("a non-first pipeline stage requires an activation")
    output = model(stage_input, labels if ctx.is_last_stage else None)
    if ctx.is_last_stage:
        # Scaled losses add up to the loss of one logical large batch.
        output = output / num_microbatches
        losses.append(output.detach())
    return output


def _backward_step(input_tensor, output_tensor, output_gradient, ctx):
    with _nvtx(f"backward stage {ctx.pp_rank}"):
        return _backward_step_impl(input_tensor, output_tensor, output_gradient, ctx)


def _backward_step_impl(input_tensor, output_tensor, output_gradient, ctx):
    if ctx.is_last_stage:
        torch.autograd.backward(output_tensor)
    else:
        if output_gradient is None:
            raise RuntimeError("a non-last pipeline stage requires an output gradient")
        torch.autograd.backward(output_tensor, grad_tensors=output_gradient)
    if input_tensor is None:
        return None
    if input_tensor.grad is None:
        raise RuntimeError("pipeline input did not receive a gradient")
    return input_tensor.grad


def forward_backward_1f1b(model: nn.Module, batches: Sequence[Batch], config, device,
                          ctx: ParallelContext, before_last_backward=None) -> list[torch.Tensor]:
    """Run one 1F1B step over ``batches``; return the detached scaled losses (last stage).

    ``batches`` are ``(input_ids, labels)`` pairs, each ``[micro_batch, seq_len]``.
    ``before_last_backward`` (or else a ``before_last_backward()`` method of
    ``model``) is called right before the final microbatch's backward, where
    overlapped gradient reduction can start; the argument form receives the
    number of backwards already run in this step.
    Parity: ``nano_megatron/pipeline.py:152-224`` (validation, warm-up depth
    ``min(pp - r - 1, M)``, steady 1F1B, cool-down).
    """
    num_microbatches = len(batches)
    if num_microbatches == 0:
        raise ValueError("1F1B requires at least one microbatch")
    micro_batch_size = batches[0][0].size(0)
    expected = (micro_batch_size, config.seq_len)
    if any(tuple(x.shape) != expected or tuple(y.shape) != expected for x, y in batches):
        raise ValueError(f"every microbatch input and label must have shape {expected}")
    device = torch.device(device)
    sp = config.sequence_parallel and ctx.tp_size > 1
    seq = config.seq_len // (ctx.tp_size if sp else 1)
    p2p = _P2P(ctx, (micro_batch_size, seq, config.n_embd), config.activation_dtype, device)
    hook = before_last_backward
    if hook is None:
        method = getattr(model, "before_last_backward", None)
        hook = (lambda _prior: method()) if method is not None else None

    num_warmup = min(ctx.pp_size - ctx.pp_rank - 1, num_microbatches)
    num_steady = num_microbatches - num_warmup
    inputs: list = []
    outputs: list = []
    losses: list[torch.Tensor] = []
    batch_iter = iter(batches)
    backward_count = 0

    def run_backward(input_tensor, output_tensor, grad):
        nonlocal backward_count
        backward_count += 1
        if hook is not None and backward_count == num_microbatches:
            hook(num_microbatches - 1)
        return _backward_step(input_tensor, output_tensor, grad, ctx)

    def recv_forward():
        return None if ctx.is_first_stage else p2p.exchange(recv_prev=True)[0]

    for _ in range(num_warmup):
        hidden = recv_forward()
        output = _forward_step(model, next(batch_iter), hidden, losses, num_microbatches, ctx)
        if not ctx.is_last_stage:
            p2p.exchange(send_next=output)
        inputs.append(hidden)
        outputs.append(output)

    # Steady state: each forward is followed by one backward. The activation
    # for the next forward is received in the same batched exchange that sends
    # this backward's input gradient (and the output gradient arrives with the
    # forward's send), so adjacent stages always post matching pairs.
    hidden = recv_forward() if num_steady > 0 else None
    for k in range(num_steady):
        output = _forward_step(model, next(batch_iter), hidden, losses, num_microbatches, ctx)
        grad = None if ctx.is_last_stage else p2p.exchange(send_next=output, recv_next=True)[1]
        inputs.append(hidden)
        outputs.append(output)
        input_grad = run_backward(inputs.pop(0), outputs.pop(0), grad)
        last = k == num_steady - 1
        if ctx.is_first_stage:
            hidden = None
        elif last:
            p2p.exchange(send_prev=input_grad)
        else:
            hidden = p2p.exchange(send_prev=input_grad, recv_prev=True)[0]

    for _ in range(num_warmup):
        input_tensor, output_tensor = inputs.pop(0), outputs.pop(0)
        grad = None if ctx.is_last_stage else p2p.exchange(recv_next=True)[1]
        input_grad = run_backward(input_tensor, output_tensor, grad)
        if not ctx.is_first_stage:
            p2p.exchange(send_prev=input_grad)

    p2p.drain()
    return losses
