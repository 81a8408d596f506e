"""Distributed correctness matrix: every TP x PP x DP (x SP, recompute) config
must reproduce the single-process model.

Each rank builds the unsharded oracle from seed 0, runs it over the
concatenation of every DP replica's microbatches, loads its own slice of the
oracle weights, runs real 1F1B + gradient finalization over Gloo, and compares:
activation shapes, loss, every reassembled gradient, the logical gradient
norm and the clipped gradients against ``torch.nn.utils.clip_grad_norm_``,
parameters after one SGD step (linear, so synchronization bugs are not hidden
by Adam's sign-like first step), and rank-aware initialization sync.
DP replicas get different data on purpose, so a missing or unaveraged DP
reduction fails the gradient comparison.

    python -m tests.test_parallel_matrix --tp 2 --pp 2 --sequence-parallel
    python -m tests.test_parallel_matrix --matrix

Processes use a file rendezvous. The harness waits for a clean exit with a
bounded timeout and reports timeouts, crashes and mismatches separately.
"""

from __future__ import annotations

import argparse
import os
import queue
import tempfile
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nano_megatron_b200.models import GPT, GPTConfig
from nano_megatron_b200.parallel import init_parallel
from nano_megatron_b200.models.functional import set_grad_observer
from nano_megatron_b200.parallel.grads import (GradBucketer, clip_grad_norm, finalize_gradients,
                                               synchronize_model_parameters)
from nano_megatron_b200.parallel.pipeline import forward_backward_1f1b
from tests.oracle import full_model, gather_tensor, parallel_model

TOL = dict(rtol=1e-4, atol=1e-5)


def make_batches(config, micro_bs, count, seed):
    gen = torch.Generator().manual_seed(seed)
    shape = (micro_bs, config.seq_len)
    return [(torch.randint(0, config.vocab_size, shape, generator=gen),
             torch.randint(0, config.vocab_size, shape, generator=gen)) for _ in range(count)]


def run_full(config, batches):
    model = full_model(config)
    total = 0.0
    for x, y in batches:
        loss = model(x, y) / len(batches)
        loss.backward()
        total = total + loss.detach()
    return model, total


def full_name(name, layer_offset, tied_split):
    if name.startswith("layers."):
        _, idx, rest = name.split(".", 2)
        return f"layers.{int(idx) + layer_offset}.{rest}"
    if tied_split and name == "lm_head.weight":
        return "embedding.weight"
    return name


def equal_across(tensor, group):
    parts = [torch.empty_like(tensor) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, tensor.contiguous(), group=group)
    return all(torch.equal(parts[0], p) for p in parts[1:])


def check_init_sync(config, rank, ctx, failures):
    torch.manual_seed(10_000 + rank)
    model = GPT(config, ctx)
    synchronize_model_parameters(model, ctx, tie_embeddings=config.tie_word_embeddings)
    distinct_shard = False
    for name, p in model.named_parameters():
        if ctx.dp_size > 1 and not equal_across(p.data, ctx.dp_group):
            failures.append(f"init {name}: DP replicas differ")
        if ctx.tp_size > 1:
            same = equal_across(p.data, ctx.tp_group)
            if getattr(p, "tensor_parallel_sharded", False):
                distinct_shard = distinct_shard or not same
            elif not same:
                failures.append(f"init {name}: TP-replicated values differ")
    if ctx.tp_size > 1 and not distinct_shard:
        failures.append("init: every TP shard is identical")
    if ctx.pp_size > 1 and (ctx.is_first_stage or ctx.is_last_stage):
        tied = model.embedding.weight if ctx.is_first_stage else model.lm_head.weight
        if not equal_across(tied.data, ctx.tied_group):
            failures.append("init: tied embedding copies differ across stages")


def worker(rank, world, init_file, args, results):
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        ctx = init_parallel(tp_size=args.tp, pp_size=args.pp)
        config = GPTConfig(vocab_size=args.vocab_size, n_layer=args.n_layer, n_head=args.n_head,
                           n_embd=args.n_embd, seq_len=args.seq_len, tie_word_embeddings=True,
                           sequence_parallel=args.sequence_parallel, recompute=args.recompute,
                           ffn_hidden_size=args.ffn_hidden_size)
        batches = make_batches(config, args.micro_batch_size, args.num_microbatches, 1234 + ctx.dp_rank)
        all_batches = [b for r in range(args.dp)
                       for b in make_batches(config, args.micro_batch_size, args.num_microbatches, 1234 + r)]
        full, _ = run_full(config, all_batches)
        model = parallel_model(config, full, ctx)
        model.train()

        shapes = []
        hooks = [layer.register_forward_hook(lambda _m, _i, out: shapes.append(tuple(out.shape)))
                 for layer in model.layers]
        bucketer = None
        if args.dp_bucket_bytes and ctx.dp_size > 1:
            bucketer = GradBucketer(model, ctx, bucket_bytes=args.dp_bucket_bytes)
            set_grad_observer(bucketer.observe)
        losses = forward_backward_1f1b(model, batches, config, "cpu", ctx,
                                       before_last_backward=bucketer.before_last_backward if bucketer else None)
        for h in hooks:
            h.remove()
        if bucketer is not None:
            started_in_backward = sum(bucketer.started)
            bucketer.finish()
            set_grad_observer(None)
            if args.num_microbatches > 1 and started_in_backward == 0:
                failures_pre = ["bucketer: no bucket started during the last backward"]
            else:
                failures_pre = []
        else:
            failures_pre = []
        finalize_gradients(model, ctx, tie_embeddings=True,
                           sequence_parallel=config.sequence_parallel, skip_data_parallel=bucketer is not None)

        failures = list(failures_pre)
        seq = config.seq_len // (args.tp if config.sequence_parallel else 1)
        if not shapes:
            failures.append("no layer forward was seen by the forward hooks")
        if any(s[0] != seq * args.micro_batch_size for s in shapes):
            failures.append(f"activation rows {[s[0] for s in shapes]} != {seq * args.micro_batch_size}")
        if ctx.is_last_stage:
            _, local_loss = run_full(config, batches)
            got = torch.stack(losses).sum()
            if not torch.allclose(got, local_loss, **TOL):
                failures.append(f"loss {got.item():.6f} != {local_loss.item():.6f}")

        ref_params = dict(full.named_parameters())
        offset = ctx.pp_rank * (config.n_layer // args.pp)

        def compare(label, getter):
            for name, p in model.named_parameters():
                ref = getter(ref_params.get(full_name(name, offset, args.pp > 1)))
                got = gather_tensor(name, p.grad if label != "param" else p.data, ctx)
                if ref is None:
                    failures.append(f"{label} {name}: no reference")
                elif not torch.allclose(got, ref, **TOL):
                    failures.append(f"{label} {name}: max_abs_err={(got - ref).abs().max().item():.3e}")

        compare("grad", lambda p: None if p is None else p.grad)
        ref_norm = torch.nn.utils.clip_grad_norm_(full.parameters(), args.clip)
        norm = clip_grad_norm(model, ctx, args.clip, tie_embeddings=True)
        if not torch.allclose(norm.float(), ref_norm.float(), **TOL):
            failures.append(f"grad norm {norm.item():.6f} != {ref_norm.item():.6f}")
        compare("clipped grad", lambda p: None if p is None else p.grad)

        torch.optim.SGD(full.parameters(), lr=1e-3).step()
        torch.optim.SGD(model.parameters(), lr=1e-3).step()
        compare("param", lambda p: None if p is None else p.data)

        check_init_sync(config, rank, ctx, failures)
        results.put((rank, ctx.describe(), failures))
    finally:
        dist.destroy_process_group()


def run_config(args, verbose=True) -> bool:
    world = args.tp * args.pp * args.dp
    mpctx = mp.get_context("spawn")
    results = mpctx.Queue()
    with tempfile.TemporaryDirectory() as tmp:
        init_file = os.path.join(tmp, "rendezvous")
        procs = [mpctx.Process(target=worker, args=(r, world, init_file, args, results))
                 for r in range(world)]
        for p in procs:
            p.start()
        got = []
        deadline = time.monotonic() + args.timeout
        while len(got) < world and time.monotonic() < deadline:
            try:
                got.append(results.get(timeout=0.2))
            except queue.Empty:
                if any(p.exitcode not in (None, 0) for p in procs):
                    break
        # Ranks that reported are only tearing down; give them a generous bound.
        for p in procs:
            p.join(timeout=max(5.0, deadline - time.monotonic()))
        timed_out = [p for p in procs if p.is_alive()]
        for p in timed_out:
            p.terminate()
            p.join()
        crashed = [p.exitcode for p in procs if p not in timed_out and p.exitcode != 0]
    got.sort()
    mismatches = sum(len(f) for _, _, f in got)
    if verbose:
        for _, desc, fails in got:
            print(f"  {desc}")
            for f in fails:
                print(f"      FAIL {f}")
    ok = mismatches == 0 and not crashed and not timed_out and len(got) == world
    label = (f"tp={args.tp} pp={args.pp} dp={args.dp} M={args.num_microbatches} "
             f"sp={int(args.sequence_parallel)} rc={int(args.recompute)}"
             f"{' dp-buckets' if args.dp_bucket_bytes else ''}")
    detail = "" if ok else (f"  ({mismatches} mismatches, {len(crashed)} crashes, "
                            f"{len(timed_out)} timeouts, {world - len(got)} missing)")
    print(f"{'PASS' if ok else 'FAIL'}  {label}{detail}", flush=True)
    return ok


MATRIX = [  # (tp, pp, dp, microbatches, sequence_parallel, recompute)
    (1, 1, 1, 4, False, False), (2, 1, 1, 4, False, False), (4, 1, 1, 4, False, False),
    (1, 2, 1, 4, False, False), (2, 2, 1, 4, False, False), (1, 4, 1, 4, False, False),
    (1, 4, 1, 1, False, False), (1, 1, 2, 4, False, False), (2, 1, 2, 4, False, False),
    (1, 2, 2, 4, False, False), (2, 2, 2, 2, False, False), (2, 1, 1, 4, True, False),
    (4, 1, 1, 4, True, False), (2, 2, 1, 4, True, False), (2, 2, 2, 2, True, False),
    (2, 2, 1, 2, True, True),
]
# DP configs again with the gradient bucketer (small buckets: several per stage)
MATRIX_BUCKETS = [(1, 1, 2, 4, False, False), (2, 2, 2, 2, True, False), (1, 2, 2, 1, False, False)]


def build_parser():
    p = argparse.ArgumentParser()
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--pp", type=int, default=1)
    p.add_argument("--dp", type=int, default=1)
    p.add_argument("--matrix", action="store_true")
    p.add_argument("--num-microbatches", type=int, default=4)
    p.add_argument("--micro-batch-size", type=int, default=2)
    p.add_argument("--n-layer", type=int, default=4)
    p.add_argument("--n-head", type=int, default=4)
    p.add_argument("--n-embd", type=int, default=64)
    p.add_argument("--ffn-hidden-size", type=int, default=None)
    p.add_argument("--vocab-size", type=int, default=128)
    p.add_argument("--seq-len", type=int, default=16)
    p.add_argument("--clip", type=float, default=0.25)
    p.add_argument("--sequence-parallel", action="store_true")
    p.add_argument("--recompute", action="store_true")
    p.add_argument("--timeout", type=float, default=180.0)
    p.add_argument("--dp-bucket-bytes", type=int, default=0,
                   help="reduce DP gradients with the bucketer, buckets of this many bytes")
    return p


def main():
    args = build_parser().parse_args()
    if not args.matrix:
        raise SystemExit(0 if run_config(args) else 1)
    results = []
    for buckets, configs in ((0, MATRIX), (4096, MATRIX_BUCKETS)):
        for tp, pp, dp, m, sp, rc in configs:
            args.tp, args.pp, args.dp, args.num_microbatches = tp, pp, dp, m
            args.sequence_parallel, args.recompute, args.dp_bucket_bytes = sp, rc, buckets
            results.append(run_config(args, verbose=False))
    print(f"\n{sum(results)}/{len(results)} configurations passed")
    raise SystemExit(0 if all(results) else 1)


@pytest.mark.distributed
@pytest.mark.parametrize("tp,pp,dp,sp,rc,ffn,buckets", [
    (2, 1, 1, False, False, None, 0),
    (2, 2, 1, True, False, 48, 0),
    (2, 2, 2, True, True, None, 0),
    (1, 2, 2, False, False, None, 0),
    (2, 2, 2, True, False, None, 2048),
])
def test_distributed_matrix(tp, pp, dp, sp, rc, ffn, buckets):
    args = build_parser().parse_args(["--n-embd=32", "--vocab-size=64", "--seq-len=8",
                                      "--micro-batch-size=1", "--num-microbatches=2"])
    args.tp, args.pp, args.dp, args.sequence_parallel, args.recompute = tp, pp, dp, sp, rc
    args.ffn_hidden_size, args.dp_bucket_bytes = ffn, buckets
    assert run_config(args, verbose=True)


if __name__ == "__main__":
    main()
