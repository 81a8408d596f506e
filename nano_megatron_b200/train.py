"""Training loop and ``torchrun`` command line.

    torchrun --nproc-per-node=4 -m nano_megatron_b200.train --tp 2 --pp 2 --sequence-parallel

:class:`Trainer` is the public training API (model, optimizer, one
``train_step`` per global batch); the CLI wires it to a token stream and to
rank-local checkpoints. Flags and defaults are those of the reference
(``nano_megatron/train.py:182-208``) plus ``--ffn-hidden-size``,
``--rope-theta``, ``--untie-embeddings``, ``--init-std``, ``--init-device``,
``--timing``, ``--no-fused-tp``, ``--load-reference`` and ``--save-format``.
"""

from __future__ import annotations

import argparse
import os
import random
import time
from pathlib import Path

import torch
import torch.distributed as dist

from .models import GPT, GPTConfig
from .optim import FusedAdamW
from .parallel import ParallelContext, init_parallel
from .models.functional import set_grad_observer
from .parallel.grads import (GradBucketer, clip_coefficient, clip_grad_norm, finalize_gradients,
                             grad_norm_squared, synchronize_model_parameters)
from .parallel.pipeline import forward_backward_1f1b
from .utils.checkpoint import (export_reference_checkpoint, import_reference_checkpoint, load_checkpoint,
                               reference_config_problems, save_checkpoint)
from .utils.data import TokenStream, synthetic_batches


class Trainer:
    """One model stage, its optimizer and the per-step training procedure."""

    def __init__(self, config: GPTConfig, ctx: ParallelContext, device, *, lr: float = 3e-4,
                 clip: float = 1.0, seed: int = 0, init_device=None, fused_tp: bool = True,
                 dp_bucket_mb: float = 128.0):
        self.config, self.ctx, self.clip = config, ctx, clip
        self.device = torch.device(device)
        if self.device.type == "cuda":
            ctx.resources["fused_tp"] = fused_tp
        # TP shards and pipeline stages draw different values; DP replicas of a
        # shard draw the same, and replicated parameters are broadcast below.
        model_seed = seed + ctx.tp_size * ctx.pp_rank + ctx.tp_rank
        random.seed(model_seed)
        torch.manual_seed(model_seed)
        if init_device is not None and torch.device(init_device).type == "cuda":
            torch.cuda.manual_seed(model_seed)
            self.model = GPT(config, ctx, device=self.device)
        else:
            self.model = GPT(config, ctx).to(self.device)
        synchronize_model_parameters(self.model, ctx, tie_embeddings=config.tie_word_embeddings)
        self.optimizer = FusedAdamW(self.model, lr=lr)
        # Data-parallel averaging bucket by bucket during the last backward, on
        # a communication stream beside the compute stream. The fused TP
        # kernels and the averaging kernel claim their work dynamically, so
        # neither needs its whole grid resident to finish.
        self.bucketer = None
        if ctx.dp_size > 1 and dp_bucket_mb > 0 and getattr(self.model, "flat_buffers", None) is not None:
            reducer = None
            if self.device.type == "cuda":
                # our NVLink averaging kernel over a symmetric gradient buffer
                from .ops.dp_reduce import DPWorkspace
                self.dp_workspace = DPWorkspace(ctx, self.model.flat_buffers)
                reducer = self.dp_workspace.all_reduce_avg
            self.bucketer = GradBucketer(self.model, ctx, bucket_bytes=int(dp_bucket_mb * (1 << 20)),
                                         overlap=True, reducer=reducer)
            set_grad_observer(self.bucketer.observe)

    def to_device(self, batches):
        return [(x.to(self.device, non_blocking=True), y.to(self.device, non_blocking=True))
                for x, y in batches]

    def check_kernel_status(self) -> None:
        """Raise if a kernel of this rank reported an error (bounded wait ran out,
        token out of range, ...) since the last check; one device sync on CUDA."""
        if self.device.type == "cuda":
            from . import ops
            ops.cuda_ops().check_status(self.device)

    def train_step(self, batches) -> torch.Tensor | None:
        """Forward, backward, gradient sync, clip and AdamW over one global batch.

        ``batches`` is a list of ``(input_ids, labels)`` microbatches (host or
        device). Returns the DP-averaged loss as a device scalar on the last
        pipeline stage's TP rank 0, None on every other rank.
        """
        cfg, ctx, model = self.config, self.ctx, self.model
        self.optimizer.zero_grad()
        batches = self.to_device(batches)
        bucketer = self.bucketer
        losses = forward_backward_1f1b(model, batches, cfg, self.device, ctx,
                                       before_last_backward=bucketer.before_last_backward if bucketer else None)
        if bucketer is not None:
            bucketer.finish()
        finalize_gradients(model, ctx, tie_embeddings=cfg.tie_word_embeddings,
                           sequence_parallel=cfg.sequence_parallel, skip_data_parallel=bucketer is not None)
        if self.device.type == "cuda":
            # Norm on the device, coefficient applied inside the fused AdamW.
            if self.clip < 0:
                raise ValueError(f"max_norm must be non-negative, got {self.clip}")
            norm = grad_norm_squared(model, ctx, tie_embeddings=cfg.tie_word_embeddings).sqrt()
            self.optimizer.step(grad_scale=clip_coefficient(norm, self.clip))
        else:
            clip_grad_norm(model, ctx, self.clip, tie_embeddings=cfg.tie_word_embeddings)
            self.optimizer.step()
        if not (ctx.is_last_stage and ctx.tp_rank == 0):
            return None
        loss = torch.stack(losses).sum()
        if ctx.dp_size > 1:
            dist.all_reduce(loss, group=ctx.dp_group)
            loss /= ctx.dp_size
        return loss


def config_from_args(args) -> GPTConfig:
    return GPTConfig(
        vocab_size=args.vocab_size, n_layer=args.n_layer, n_head=args.n_head,
        n_embd=args.n_embd, seq_len=args.seq_len,
        tie_word_embeddings=not args.untie_embeddings,
        sequence_parallel=args.sequence_parallel, recompute=args.recompute,
        compute_dtype=args.dtype, ffn_hidden_size=args.ffn_hidden_size,
        rope_theta=args.rope_theta, init_std=args.init_std)


def _parse_fault(spec: str | None):
    """``RANK:STEP:MODE`` -> (rank, step, mode); host-side fault injection for tests."""
    if not spec:
        return None
    rank, step, mode = spec.split(":")
    if mode not in ("leave", "raise", "hang", "vanish"):
        raise ValueError(f"--inject-fault mode {mode!r}: use leave, raise, hang or vanish")
    return int(rank), int(step), mode


def _inject(fault, rank: int, step: int, watch) -> None:
    """Make this rank fail between steps, the way a real job can: announce and
    exit cleanly (leave), raise (raise), stop without a word for a bounded time
    (hang), or die without a word (vanish)."""
    if fault is None or fault[0] != rank or fault[1] != step:
        return
    mode = fault[2]
    if mode == "leave":
        if watch is not None:
            watch.leave(f"left on request before step {step}")
        os._exit(0)
    if mode == "raise":
        raise RuntimeError(f"injected fault before step {step}")
    if mode == "hang":
        time.sleep(600)  # the harness kills it long before this ends
        os._exit(4)
    os._exit(3)  # vanish: like a process killed by a signal


def train(args):
    from datetime import timedelta

    from .utils.health import PeerLost, PeerWatch

    if (args.backend == "nccl") != (args.device == "cuda"):
        raise ValueError("use gloo with cpu or nccl with cuda")
    if args.backend == "nccl":
        torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group(backend=args.backend, timeout=timedelta(seconds=args.pg_timeout))
    rank, world = dist.get_rank(), dist.get_world_size()
    if world != args.tp * args.pp * args.dp:
        raise ValueError(f"torchrun world size {world} != tp * pp * dp = {args.tp * args.pp * args.dp}")
    watch = PeerWatch(rank, world, timeout=args.peer_timeout) if args.peer_timeout > 0 else None
    fault = _parse_fault(args.inject_fault)
    try:
        _train_loop(args, rank, watch, fault)
    except PeerLost as exc:
        watch.leave(f"stopped because {exc}")
        raise
    except BaseException as exc:
        if watch is not None:
            watch.leave(f"{type(exc).__name__}: {exc}")
        raise
    dist.barrier()
    dist.destroy_process_group()


def _train_loop(args, rank, watch, fault):
    ctx = init_parallel(tp_size=args.tp, pp_size=args.pp)
    device = (torch.device("cuda", int(os.environ["LOCAL_RANK"])) if args.device == "cuda"
              else torch.device(args.device))
    config = config_from_args(args)
    if args.save and args.save_format == "reference" and reference_config_problems(config):
        raise ValueError("--save-format reference: " + "; ".join(reference_config_problems(config)))
    trainer = Trainer(config, ctx, device, lr=args.lr, clip=args.clip, seed=args.seed,
                      init_device=args.init_device, fused_tp=not args.no_fused_tp,
                      dp_bucket_mb=args.dp_bucket_mb)
    stream = (TokenStream(args.data, dtype=args.data_dtype, seq_len=config.seq_len,
                          dp_rank=ctx.dp_rank, dp_size=ctx.dp_size) if args.data else None)
    training_state = {"lr": args.lr, "clip": args.clip, "micro_batch_size": args.micro_batch_size,
                      "num_microbatches": args.num_microbatches}
    # --load resumes this implementation's checkpoints, --load-reference a step
    # directory saved by the reference implementation (same layout, torch AdamW state)
    resume, loader = ((args.load, load_checkpoint) if args.load else
                      (args.load_reference, import_reference_checkpoint))
    start_step, loaded_extra = (loader(resume, trainer.model, trainer.optimizer, ctx, data=stream,
                                       map_location=device)
                                if resume else (0, {}))
    if loaded_extra and loaded_extra != training_state:
        raise RuntimeError(f"checkpoint training configuration mismatch: saved={loaded_extra}, "
                           f"current={training_state}")
    if rank == 0:
        total = sum(p.numel() for p in trainer.model.parameters())
        print(f"{ctx.describe()}\nlocal params: {total / 1e6:.2f}M  schedule: 1f1b\n", flush=True)

    poller = None
    if device.type == "cuda":
        from .ops.cuda import StatusPoller
        poller = StatusPoller(device)
    timing = args.timing and device.type == "cuda"
    for step in range(start_step, args.steps):
        _inject(fault, rank, step, watch)
        if watch is not None:
            watch.enter_step()  # raises PeerLost before any kernel of this step is launched
        t0 = time.perf_counter()
        if timing:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        if stream is None:
            batches = synthetic_batches(config, args.micro_batch_size, args.num_microbatches,
                                        step, ctx.dp_rank)
        else:
            batches = [stream.next_batch(args.micro_batch_size) for _ in range(args.num_microbatches)]
        loss = trainer.train_step(batches)
        if poller is not None:
            poller.poll()  # kernel errors (bounded waits, token ids) surface without a device sync
        if timing:
            ev1.record()
            ev1.synchronize()
            elapsed = torch.tensor(ev0.elapsed_time(ev1) / 1e3, device=device)
            dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)  # device time, max over ranks
            elapsed = elapsed.item()
        else:
            elapsed = time.perf_counter() - t0
        if loss is not None and ctx.dp_rank == 0:
            tokens = args.micro_batch_size * args.num_microbatches * config.seq_len * ctx.dp_size
            print(f"step {step:3d} | loss {loss.item():.4f} | {elapsed * 1e3:6.1f} ms | "
                  f"{tokens / elapsed:8.0f} tok/s", flush=True)
        next_step = step + 1
        if args.save and (next_step == args.steps
                          or (args.save_every > 0 and next_step % args.save_every == 0)):
            if poller is not None:
                poller.final()  # never checkpoint state that a failed kernel produced
            saver = export_reference_checkpoint if args.save_format == "reference" else save_checkpoint
            saver(Path(args.save) / f"step_{next_step:08d}", trainer.model, trainer.optimizer, ctx,
                  step=next_step, data=stream, extra=training_state)
    if poller is not None:
        poller.final()


def build_parser():
    p = argparse.ArgumentParser(description="Train a GPT with TP + SP + PP + DP.")
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--pp", type=int, default=1)
    p.add_argument("--dp", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--num-microbatches", type=int, default=4)
    p.add_argument("--micro-batch-size", type=int, default=4)
    p.add_argument("--n-layer", type=int, default=4)
    p.add_argument("--n-head", type=int, default=4)
    p.add_argument("--n-embd", type=int, default=128)
    p.add_argument("--vocab-size", type=int, default=256)
    p.add_argument("--seq-len", type=int, default=32)
    p.add_argument("--sequence-parallel", action="store_true")
    p.add_argument("--recompute", action="store_true")
    p.add_argument("--dtype", choices=["float32", "bfloat16"], default="float32")
    p.add_argument("--lr", type=float, default=3e-4)
    p.add_argument("--clip", type=float, default=1.0)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--device", default="cpu")
    p.add_argument("--backend", default="gloo", choices=["gloo", "nccl"])
    p.add_argument("--data", help="raw pre-tokenized uint16/uint32 file")
    p.add_argument("--data-dtype", choices=["uint16", "uint32"], default="uint16")
    p.add_argument("--save", help="directory for rank-local checkpoint steps")
    p.add_argument("--save-every", type=int, default=0, help="0 saves only the final step")
    p.add_argument("--load", help="exact checkpoint step directory to resume")
    p.add_argument("--load-reference", default=None,
                   help="resume a step directory saved by the reference implementation (nano_megatron)")
    p.add_argument("--save-format", choices=["native", "reference"], default="native",
                   help="write --save steps in this implementation's format or in one the reference "
                        "implementation's --load resumes")
    # extensions
    p.add_argument("--ffn-hidden-size", type=int, default=None, help="SwiGLU width (default 4*n_embd)")
    p.add_argument("--rope-theta", type=float, default=10000.0)
    p.add_argument("--untie-embeddings", action="store_true")
    p.add_argument("--init-std", type=float, default=0.02)
    p.add_argument("--init-device", default=None,
                   help="initialize weights directly on this device (e.g. cuda) instead of CPU")
    p.add_argument("--timing", action="store_true", help="CUDA-event step time, max over ranks")
    p.add_argument("--dp-bucket-mb", type=float, default=128.0,
                   help="data-parallel gradient bucket size in MiB, reduced during the last backward "
                        "(0: one all-reduce of the whole gradient buffer after backward)")
    p.add_argument("--no-fused-tp", action="store_true",
                   help="use NCCL collectives instead of the fused TP kernels")
    p.add_argument("--peer-timeout", type=float, default=300.0,
                   help="seconds a rank waits at a step boundary for a silent peer before raising "
                        "PeerLost (0 disables the host-side peer watch)")
    p.add_argument("--pg-timeout", type=float, default=1800.0,
                   help="process-group timeout in seconds: a collective whose peers never arrive "
                        "ends with an error after this long")
    p.add_argument("--inject-fault", default=None, help=argparse.SUPPRESS)  # RANK:STEP:MODE (tests)
    return p


def main(argv=None):
    args = build_parser().parse_args(argv)
    if args.steps < 0 or args.save_every < 0:
        raise ValueError("steps and save-every must be non-negative")
    if args.num_microbatches <= 0 or args.micro_batch_size <= 0:
        raise ValueError("num-microbatches and micro-batch-size must be positive")
    if args.load and args.load_reference:
        raise ValueError("--load and --load-reference are exclusive")
    train(args)


if __name__ == "__main__":
    main()
