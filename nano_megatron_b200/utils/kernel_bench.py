"""Single-GPU kernel microbenchmarks (also the small cases used for ncu captures).

    python -m nano_megatron_b200.utils.kernel_bench attention --seq 8192 --heads 32 [--sdpa]
    python -m nano_megatron_b200.utils.kernel_bench gemm --shapes 8192x12288x4096 [--cublas]

Times each op with CUDA events on the current stream after warm-up and prints
one JSON line per case. ``--iters 1 --warmup 1`` gives a capture-sized run.
Attention FLOPs count causal attention as ``4 * S^2 * d * heads / 2`` forward
and 2.5x that backward.
"""

from __future__ import annotations

import argparse
import json

import torch


def _time(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) / iters


def bench_attention(args):
    from ..ops import cuda as K
    from ..ops import reference as R
    dev = torch.device("cuda")
    S, b, h, d = args.seq, args.batch, args.heads, 128
    cos, sin = R.rope_cache(S, d, 500000.0, dev)
    qkv = torch.randn(S * b, 3 * h * d, device=dev).bfloat16()
    o, saved = K.attention(qkv, b, h, d, cos, sin)
    do = torch.randn_like(o)
    flops = 4.0 * S * S * h * d / 2 * b
    fwd = _time(lambda: K.attention(qkv, b, h, d, cos, sin), args.iters, args.warmup)
    bwd = _time(lambda: K.attention_bwd(do, saved, b, h, d, cos, sin), args.iters, args.warmup)
    K.check_status(dev)
    out = {"op": "attention", "impl": "ours", "S": S, "batch": b, "heads": h, "fwd_ms": round(fwd, 3),
           "bwd_ms": round(bwd, 3), "fwd_tflops": round(flops / fwd / 1e9, 1),
           "bwd_tflops": round(2.5 * flops / bwd / 1e9, 1)}
    print(json.dumps(out), flush=True)
    if args.sdpa:
        import torch.nn.functional as F
        q = torch.randn(b, h, S, d, device=dev, dtype=torch.bfloat16, requires_grad=True)
        k = torch.randn_like(q, requires_grad=True)
        v = torch.randn_like(q, requires_grad=True)
        g = torch.randn_like(q)
        fwd = _time(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True), args.iters, args.warmup)
        both = _time(lambda: torch.autograd.grad(F.scaled_dot_product_attention(q, k, v, is_causal=True),
                                                 (q, k, v), g), args.iters, args.warmup)
        print(json.dumps({"op": "attention", "impl": "torch sdpa (default backend)", "S": S, "heads": h,
                          "fwd_ms": round(fwd, 3), "bwd_ms": round(both - fwd, 3),
                          "fwd_tflops": round(flops / fwd / 1e9, 1),
                          "bwd_tflops": round(2.5 * flops / (both - fwd) / 1e9, 1)}), flush=True)


def bench_gemm(args):
    from ..ops import cuda as K
    dev = torch.device("cuda")
    for shape in args.shapes:
        M, N, Kd = (int(x) for x in shape.split("x"))
        a = torch.randn(M, Kd, device=dev).bfloat16()
        w = torch.randn(Kd, N, device=dev).bfloat16()
        wt = w.t().contiguous()
        dy = torch.randn(M, N, device=dev).bfloat16()
        acc = torch.zeros(Kd, N, device=dev)
        flops = 2.0 * M * N * Kd
        res = {"nn": _time(lambda: K.mm_nn(a, w), args.iters, args.warmup),
               "nt": _time(lambda: K.mm_nt(a, wt), args.iters, args.warmup),
               "tn_acc": _time(lambda: K.mm_tn_acc(a, dy, acc), args.iters, args.warmup)}
        line = {"op": "gemm", "M": M, "N": N, "K": Kd,
                **{f"{k}_tflops": round(flops / v / 1e9, 1) for k, v in res.items()}}
        if args.cublas:
            line["cublas_nn_tflops"] = round(flops / _time(lambda: a @ w, args.iters, args.warmup) / 1e9, 1)
        print(json.dumps(line), flush=True)


def main(argv=None):
    p = argparse.ArgumentParser()
    sub = p.add_subparsers(dest="what", required=True)
    pa = sub.add_parser("attention")
    pa.add_argument("--seq", type=int, default=8192)
    pa.add_argument("--batch", type=int, default=1)
    pa.add_argument("--heads", type=int, default=32)
    pa.add_argument("--sdpa", action="store_true", help="also time torch scaled_dot_product_attention")
    pg = sub.add_parser("gemm")
    pg.add_argument("--shapes", nargs="+", default=["8192x12288x4096", "8192x4096x14336"])
    pg.add_argument("--cublas", action="store_true", help="also time torch.matmul (cuBLAS)")
    for sp in (pa, pg):
        sp.add_argument("--iters", type=int, default=5)
        sp.add_argument("--warmup", type=int, default=2)
    args = p.parse_args(argv)
    {"attention": bench_attention, "gemm": bench_gemm}[args.what](args)


if __name__ == "__main__":
    main()
