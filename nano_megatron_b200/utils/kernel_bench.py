"""Single-GPU kernel microbenchmarks (also the small cases used for ncu captures).

    python -m nano_megatron_b200.utils.kernel_bench attention --seq 8192 --heads 32 [--sdpa]
    python -m nano_megatron_b200.utils.kernel_bench gemm --shapes 8192x12288x4096 [--cublas]
    python -m nano_megatron_b200.utils.kernel_bench memory [--rows 8192 --hidden 4096 --ffn 14336]
    python -m nano_megatron_b200.utils.kernel_bench mma

``mma`` reports the cycles one tcgen05.mma (M=128, bf16 in, fp32 out) takes
in a long chain on one SM, for N = 64, 128, 256 and the A operand from shared
memory (SS) or TMEM (TS), against N/2 cycles of arithmetic at the dense bf16
rate (8192 FLOP per cycle per SM).

Times each op with CUDA events on the current stream after warm-up and prints
one JSON line per case. ``--iters 1 --warmup 1`` gives a capture-sized run.
Attention FLOPs count causal attention as ``4 * S^2 * d * heads / 2`` forward
and 2.5x that backward. ``memory`` times the memory-bound kernels at the
headline shapes (one microbatch of 8192 tokens at tp1) and reports the
algorithmic bytes each must move (every input read once, every output
written once) over its time, against the measured copy bandwidth of
``MEASURED_PEAKS.json``; every input is larger than the 126 MB L2, and the L2
is flushed between iterations by writing a 256 MB buffer (outside the timed
span).
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


def _time_flushed(fn, iters, warmup):
    """Mean time of ``fn`` with a 256 MB write between calls (outside the timing)."""
    scrub = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    for _ in range(warmup):
        fn()
    total = 0.0
    for _ in range(iters):
        scrub.fill_(1.0)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        end.synchronize()
        total += start.elapsed_time(end)
    return total / iters


def bench_memory(args):
    import os
    from ..ops import cuda as K
    from ..ops import reference as R
    dev = torch.device("cuda")
    try:
        with open(os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")) as f:
            peak, src = json.load(f)["hbm_gbs"], "hbm_gbs of measured"
    except (OSError, ValueError, KeyError):
        peak, src = 6650.0, "6.65 TB/s of fallback"
    T, H, F, heads = args.rows, args.hidden, args.ffn, args.hidden // 128
    bf = torch.bfloat16
    x = torch.randn(T, H, device=dev).to(bf)
    w = torch.rand(H, device=dev) + 0.5
    _, rstd = K.rmsnorm(x, w, 1e-6)
    dy = torch.randn_like(x)
    dw = torch.zeros(H, device=dev)
    gu = torch.randn(T, 2 * F, device=dev).to(bf)
    da = torch.randn(T, F, device=dev).to(bf)
    qkv = torch.randn(T, 3 * H, device=dev).to(bf)
    cos, sin = R.rope_cache(T, 128, 500000.0, dev)
    n = args.params
    p32, g32 = torch.randn(n, device=dev), torch.randn(n, device=dev)
    m32, v32 = torch.zeros(n, device=dev), torch.zeros(n, device=dev)
    comp = torch.empty(n, device=dev, dtype=bf)
    one = torch.ones(1, device=dev)
    V = args.vocab
    logits = torch.randn(T, V, device=dev).to(bf)
    labels = torch.randint(0, V, (T,), device=dev)
    mx, se, _, _ = K.ce_local_stats(logits, labels, 0, V)
    B2, B4 = 2, 4
    cases = [
        ("rmsnorm fwd", lambda: K.rmsnorm(x, w, 1e-6), T * H * B2 * 2 + T * B4),
        ("rmsnorm bwd", lambda: K.rmsnorm_bwd(dy, x, w, rstd, dw), T * H * B2 * 3 + T * B4),
        ("residual add + rmsnorm fwd", lambda: K.add_rmsnorm(x, dy, w, 1e-6), T * H * B2 * 4 + T * B4),
        ("rmsnorm bwd + residual gradient", lambda: K.rmsnorm_bwd(dy, x, w, rstd, dw, dres=dy),
         T * H * B2 * 4 + T * B4),
        ("swiglu fwd", lambda: K.swiglu(gu), T * F * B2 * 3),
        ("swiglu bwd", lambda: K.swiglu_bwd(da, gu), T * F * B2 * 5),
        ("rope (q and k, in place)", lambda: K.C.rope_inplace(qkv, cos, sin, 1, heads, 128, 1.0),
         T * 2 * H * B2 * 2 + T * 64 * B4 * 2),
        ("adamw (fp32 master, moments, bf16 copy)",
         lambda: K.adamw_flat(p32, g32, m32, v32, comp, one, lr=1e-4, beta1=0.9, beta2=0.999, eps=1e-8,
                              weight_decay=0.01, step=1), n * (B4 * 4 + B4 * 3 + B2)),
        ("cross-entropy grad (softmax - onehot, bf16 logits)",
         lambda: K.ce_grad(logits, labels, 0, mx, se, one, bf), T * V * B2 * 2),
    ]
    for name, fn, nbytes in cases:
        ms = _time_flushed(fn, args.iters, args.warmup)
        gbs = nbytes / ms / 1e6
        print(json.dumps({"op": name, "ms": round(ms, 4), "bytes": int(nbytes), "GB/s": round(gbs, 1),
                          "frac_of_peak": round(gbs / peak, 3), "peak": src}), flush=True)
    K.check_status(dev)


def bench_mma(args):
    from nano_megatron_b200 import _C
    from nano_megatron_b200.ops import cuda as K

    dev = torch.device("cuda", 0)
    err = K.status_word(dev)
    for ts in (False, True):
        for n in (64, 128, 256):
            cyc = _C.mma_cycles(n, ts, args.chain, err)
            ideal = 128 * n * 16 * 2 / 8192
            print(json.dumps({"op": "tcgen05.mma", "M": 128, "N": n, "K": 16, "A": "tmem" if ts else "smem",
                              "cycles": round(cyc, 1), "arith_cycles": ideal, "efficiency": round(ideal / cyc, 3)}),
                  flush=True)
    K.check_status(dev)


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
    pm = sub.add_parser("memory")
    pm.add_argument("--rows", type=int, default=8192)
    pm.add_argument("--hidden", type=int, default=4096)
    pm.add_argument("--ffn", type=int, default=14336)
    pm.add_argument("--vocab", type=int, default=32064, help="LM-head shard width for the CE gradient")
    pm.add_argument("--params", type=int, default=1 << 28, help="parameters in the AdamW buffer")
    pq = sub.add_parser("mma")
    pq.add_argument("--chain", type=int, default=2048, help="products per measured chain")
    for sp in (pa, pg, pm):
        sp.add_argument("--iters", type=int, default=5)
        sp.add_argument("--warmup", type=int, default=2)
    args = p.parse_args(argv)
    {"attention": bench_attention, "gemm": bench_gemm, "memory": bench_memory, "mma": bench_mma}[args.what](args)


if __name__ == "__main__":
    main()
