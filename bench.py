"""Training-throughput benchmark of the named configurations (tokens/s per box).

    python bench.py --gpus 1 --steps K --warmup W                  # this framework
    torchrun --nproc-per-node 8 bench.py --gpus 8 --steps K --warmup W
    python bench.py --impl reference ...                           # the reference, same config
    python bench.py --config 3 ...                                 # another named configuration

``--config 5`` (the default, the headline): Llama-3-8B shape -- vocab 128256,
hidden 4096, 32 layers, 32 heads (head_dim 128), SwiGLU ffn 14336, RoPE theta
500000, untied embeddings, seq 8192, micro-batch 1, 16 microbatches of 1F1B,
whole-block recompute. The model and the global batch (16 x 8192 tokens) are
fixed for every GPU count (strong scaling); the layout grows with N:
N=1 tp1, N=2 tp2, N=4 tp4, N=8 tp4 x pp2 (the named TP4 x PP2 + SP layout).

``--config 3``: 1.3B shape -- vocab 32000, hidden 2048, 24 layers, 16 heads,
SwiGLU ffn 5632, seq 4096, micro-batch 2, 8 microbatches, tied embeddings;
N GPUs run tp N (the named layout is tp8).

``--config 4``: 3B shape -- vocab 50304, hidden 2560, 32 layers, 20 heads,
SwiGLU ffn 6912, seq 2048, micro-batch 4, 16 microbatches per data-parallel
replica, tied embeddings; N=1 tp1, N=2 tp2, N=4 tp2 x pp2, N=8 tp2 x pp2 x dp2
(the named layout; the batch grows with the data-parallel width).

All: sequence parallelism, bf16 compute with fp32 master weights, AdamW with
clip 1.0; synthetic uniform tokens (a different seeded window per DP rank),
random N(0, 0.02) weights.

Timing: W untimed steps; then K steps bracketed by a barrier and
``torch.cuda.synchronize()`` and timed with CUDA events on the compute stream,
max over ranks (``value``, inputs staged on the device). A second K-step loop
measures the same metric end to end through the public ``Trainer.train_step``
API with per-step host->device copies from pinned memory and a device->host
read of the loss (``e2e``). Weights and activations are far larger than the
126 MB L2, so no L2 flush is needed between steps. SM clocks and throttle
reasons are sampled with ``nvidia-smi`` during the timed region.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from datetime import timedelta

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)
CONFIGS = {
    5: dict(metric="tokens/sec/box (device-timed, max over ranks) @8B-shape TP4\u00d7PP2+SP; MFU",
            label="llama3-8b-shape (V128256 H4096 L{L} A32 F14336 theta5e5 untied)",
            model=dict(vocab_size=128256, n_layer=32, n_head=32, n_embd=4096, seq_len=8192,
                       ffn_hidden_size=14336, rope_theta=500000.0),
            tied=False, recompute=True, micro_batch=1, num_microbatches=16, scaling="strong",
            layout={1: (1, 1), 2: (2, 1), 4: (4, 1), 8: (4, 2)}),
    3: dict(metric="tokens/sec/box (device-timed, max over ranks) @1.3B-shape TP8+SP; MFU",
            label="1.3b-shape (V32000 H2048 L{L} A16 F5632 tied)",
            model=dict(vocab_size=32000, n_layer=24, n_head=16, n_embd=2048, seq_len=4096,
                       ffn_hidden_size=5632, rope_theta=10000.0),
            tied=True, recompute=False, micro_batch=2, num_microbatches=8, scaling="strong",
            layout={1: (1, 1), 2: (2, 1), 4: (4, 1), 8: (8, 1)}),
    4: dict(metric="tokens/sec/box (device-timed, max over ranks) @3B-shape TP2\u00d7PP2\u00d7DP2+SP tied; MFU",
            label="3b-shape (V50304 H2560 L{L} A20 F6912 tied)",
            model=dict(vocab_size=50304, n_layer=32, n_head=20, n_embd=2560, seq_len=2048,
                       ffn_hidden_size=6912, rope_theta=10000.0),
            tied=True, recompute=False, micro_batch=4, num_microbatches=16, scaling="weak in data parallel",
            layout={1: (1, 1), 2: (2, 1), 4: (2, 2), 8: (2, 2)}),
}
CFG = CONFIGS[5]


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", type=int, choices=sorted(CONFIGS), default=5,
                   help="named configuration (5: the headline)")
    p.add_argument("--n-layer", type=int, default=None, help=argparse.SUPPRESS)  # debugging only
    p.add_argument("--breakdown", default=None, metavar="FILE",
                   help="after the timed runs, profile one more step per op class (CUDA events) "
                        "and write the per-rank breakdown to FILE (JSON, rank 0 writes)")
    return p.parse_args()


def measured_peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {"bf16_tflops_sustained": 1400.0, "bf16_tflops": 1590.0, "fallback": True}


def setup_dist(n):
    if "RANK" in os.environ:
        local = int(os.environ.get("LOCAL_RANK", 0))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(minutes=20), device_id=torch.device("cuda", local))
    else:
        if n != 1:
            raise SystemExit("--gpus > 1 needs torchrun (one process per GPU)")
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29500 + os.getpid() % 1000))
        torch.cuda.set_device(0)
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=timedelta(minutes=20),
                                device_id=torch.device("cuda", 0))
    return dist.get_rank(), dist.get_world_size(), torch.device("cuda", torch.cuda.current_device())


def max_over_ranks(x: float, device) -> float:
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_batches(vocab, seq, step, dp_rank, pin=False):
    gen = torch.Generator().manual_seed(1234 + 100_003 * step + dp_rank)
    out = []
    for _ in range(CFG["num_microbatches"]):
        x = torch.randint(0, vocab, (CFG["micro_batch"], seq), generator=gen)
        y = torch.randint(0, vocab, (CFG["micro_batch"], seq), generator=gen)
        out.append((x.pin_memory(), y.pin_memory()) if pin else (x, y))
    return out


# ------------------------------------------------------------------ our arm
def build_ours(tp, pp, device, n_layer):
    from nano_megatron_b200.models import GPTConfig
    from nano_megatron_b200.parallel import init_parallel
    from nano_megatron_b200.train import Trainer
    ctx = init_parallel(tp_size=tp, pp_size=pp)
    cfg = GPTConfig(**{**CFG["model"], "n_layer": n_layer}, tie_word_embeddings=CFG["tied"],
                    sequence_parallel=True, recompute=CFG["recompute"], compute_dtype="bfloat16")
    trainer = Trainer(cfg, ctx, device, lr=3e-4, clip=1.0, seed=0, init_device=device)

    def launches():
        from nano_megatron_b200.ops import cuda as KC
        return KC.LAUNCHES[0]

    return ctx, trainer.train_step, launches


# ------------------------------------------------------------ reference arm
def build_reference(tp, pp, device, n_layer):
    """The unmodified reference package (baseline/_ref) driven by its own public
    functions in the order of its ``train.py`` step loop. The benchmark shapes
    need settings its CLI cannot express; they are applied with its own
    classes: the SwiGLU width (its ``ParallelMLP`` hard-codes 4*H; the MLP's
    ``gate``/``up``/``down`` are replaced by its own ``ColumnParallelLinear`` /
    ``RowParallelLinear`` of the configured width), RoPE theta (its
    ``build_rope_cache`` base argument) and untied embeddings
    (``GPTConfig.tie_word_embeddings``). Parameters are created directly on the
    GPU (default-device context) instead of on the CPU and then moved."""
    ref = os.environ.get("NMB_REFERENCE_PATH") or os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "nano_megatron")):
        raise ImportError(f"reference package not found under {ref}")
    sys.path.insert(0, ref)
    from nano_megatron.grads import clip_grad_norm, finalize_gradients, synchronize_model_parameters
    from nano_megatron.model import GPT, GPTConfig, build_rope_cache
    from nano_megatron.parallel import init_parallel
    from nano_megatron.pipeline import forward_backward_1f1b
    from nano_megatron.tp_layers import ColumnParallelLinear, RowParallelLinear

    m, tied = CFG["model"], CFG["tied"]
    ctx = init_parallel(tp_size=tp, pp_size=pp)
    cfg = GPTConfig(vocab_size=m["vocab_size"], n_layer=n_layer, n_head=m["n_head"],
                    n_embd=m["n_embd"], seq_len=m["seq_len"], tie_word_embeddings=tied,
                    sequence_parallel=True, recompute=CFG["recompute"], compute_dtype="bfloat16")
    torch.manual_seed(tp * ctx.pp_rank + ctx.tp_rank)
    with torch.device(device):
        model = GPT(cfg, ctx)
        if m["ffn_hidden_size"] != 4 * m["n_embd"]:
            for layer in model.layers:
                mlp = layer.mlp
                mlp.gate = ColumnParallelLinear(cfg.n_embd, m["ffn_hidden_size"], ctx, bias=False)
                mlp.up = ColumnParallelLinear(cfg.n_embd, m["ffn_hidden_size"], ctx, bias=False)
                mlp.down = RowParallelLinear(m["ffn_hidden_size"], cfg.n_embd, ctx, bias=False)
        if m["rope_theta"] != 10000.0:
            cos, sin = build_rope_cache(cfg.seq_len, cfg.head_dim, device, base=m["rope_theta"])
            model.rope_cos, model.rope_sin = cos, sin
    synchronize_model_parameters(model, ctx, tie_embeddings=tied)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4)

    def step(batches):
        opt.zero_grad(set_to_none=True)
        batches = [(x.to(device, non_blocking=True), y.to(device, non_blocking=True)) for x, y in batches]
        losses = forward_backward_1f1b(model, batches, cfg, device, ctx)
        finalize_gradients(model, ctx, tie_embeddings=tied, sequence_parallel=True)
        clip_grad_norm(model, ctx, 1.0, tie_embeddings=tied)
        opt.step()
        if ctx.is_last_stage and ctx.tp_rank == 0:
            loss = torch.stack(losses).sum()
            if ctx.dp_size > 1:
                dist.all_reduce(loss, group=ctx.dp_group)
                loss /= ctx.dp_size
            return loss
        return None

    return ctx, step, lambda: 0


# ------------------------------------------------------------------- driver
def main():
    global CFG
    args = parse()
    CFG = CONFIGS[args.config]
    n = args.gpus
    if n not in CFG["layout"]:
        raise SystemExit(f"--gpus must be one of {sorted(CFG['layout'])}")
    tp, pp = CFG["layout"][n]
    rank, world, device = setup_dist(n)
    if world != n:
        raise SystemExit(f"world size {world} != --gpus {n}")
    n_layer = args.n_layer or CFG["model"]["n_layer"]
    local0 = int(os.environ.get("LOCAL_RANK", 0)) == 0
    try:
        build = build_ours if args.impl == "ours" else build_reference
        ctx, step, launches = build(tp, pp, device, n_layer)
    except ImportError as exc:
        if rank == 0:
            print(json.dumps({"impl": args.impl, "unavailable": f"import failed: {exc}"}), flush=True)
        dist.destroy_process_group()
        return

    vocab, seq = CFG["model"]["vocab_size"], CFG["model"]["seq_len"]
    dev_batches = [[(x.to(device), y.to(device)) for x, y in make_batches(vocab, seq, s, ctx.dp_rank)]
                   for s in range(2)]
    from nano_megatron_b200.utils.timing import ClockSampler
    try:
        for w in range(args.warmup):
            step(dev_batches[w % 2])
        torch.cuda.synchronize()
        sampler = ClockSampler(gpus=list(range(world))) if local0 else None
        dist.barrier()
        torch.cuda.synchronize()
        launches0 = launches()
        if sampler:
            sampler.__enter__()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for s in range(args.steps):
            step(dev_batches[s % 2])
        end.record()
        torch.cuda.synchronize()
        if sampler:
            sampler.__exit__(None, None, None)
        dist.barrier()
        kernel_launches = launches() - launches0
        ms = max_over_ranks(start.elapsed_time(end) / args.steps, device)
        if args.impl != "reference":  # a bounded wait that ran out or a bad token id raises here
            from nano_megatron_b200.ops import cuda as KC
            KC.check_status(device)

        # End to end through the public API: pinned host inputs, loss read back.
        host = [make_batches(vocab, seq, 100 + s, ctx.dp_rank, pin=True) for s in range(2)]
        bytes_in = sum(x.numel() * x.element_size() + y.numel() * y.element_size() for x, y in host[0])
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        bytes_out = 0
        for s in range(args.steps):
            loss = step(host[s % 2])
            if loss is not None:
                float(loss.item())
                bytes_out = loss.element_size()
        torch.cuda.synchronize()
        e2e_s = max_over_ranks((time.perf_counter() - t0) / args.steps, device)
        bytes_out = int(max_over_ranks(bytes_out, device))  # read on the loss-holding rank
    except torch.cuda.OutOfMemoryError as exc:
        if rank == 0:
            print(json.dumps({"impl": args.impl, "unavailable": f"CUDA out of memory at N={n}: "
                              f"{str(exc).splitlines()[0][:200]}"}), flush=True)
        dist.destroy_process_group()
        return

    breakdown = None
    if args.breakdown and args.impl == "ours":
        from nano_megatron_b200.utils.op_profile import OpProfile
        dist.barrier()
        with OpProfile() as prof:
            step(dev_batches[0])
        breakdown = prof.report(step_ms=ms)
        gathered = [None] * world
        dist.all_gather_object(gathered, breakdown)
        if rank == 0:
            with open(args.breakdown, "w") as f:
                json.dump({"step_ms_unprofiled": ms, "layout": f"tp{tp}pp{pp}",
                           "per_rank": gathered}, f, indent=1)

    tokens = CFG["micro_batch"] * CFG["num_microbatches"] * seq * ctx.dp_size
    value = tokens / (ms / 1e3)
    peaks = measured_peaks()
    from nano_megatron_b200.models import GPTConfig
    flops_tok = GPTConfig(**{**CFG["model"], "n_layer": n_layer},
                          tie_word_embeddings=CFG["tied"]).flops_per_token()
    mfu = value * flops_tok / (n * peaks.get("bf16_tflops_sustained", 1400.0) * 1e12)
    if rank == 0:
        clocks = sampler.summary() if sampler else {}
        line = {
            "metric": CFG["metric"], "value": round(value, 1), "unit": "tokens/s", "n_gpus": n,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2),
            "higher_is_better": True, "scaling": CFG["scaling"], "vs_baseline": None,
            "dtype": "bf16",
            "data": f"synthetic uniform tokens in [0,{vocab}), random-init N(0,0.02) weights",
            "config": {"name": f"config {args.config}", "model": CFG["label"].format(L=n_layer),
                       "global_batch": CFG["micro_batch"] * CFG["num_microbatches"] * ctx.dp_size,
                       "seq_len": seq, "micro_batch": CFG["micro_batch"],
                       "num_microbatches": CFG["num_microbatches"],
                       "parallelism": f"tp{tp}pp{pp}dp{ctx.dp_size}+sp"
                                      + ("+recompute" if CFG["recompute"] else ""),
                       "l2": "no flush: per-step working set (weights, activations) >> 126 MB L2"},
            "mfu": round(mfu, 4),
            "mfu_denominator": ("bf16_tflops_sustained of measured" if not peaks.get("fallback")
                                else "1.4 PFLOP/s of fallback"),
            "clocks": {k: clocks.get(k) for k in ("sm_mhz", "sm_max_mhz", "reasons")},
            "e2e": {"value": round(tokens / e2e_s, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": bytes_in, "d2h_bytes_per_step": bytes_out},
            "gpu_launches": kernel_launches,
        }
        if args.impl == "reference":
            line["impl"] = "reference"
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
