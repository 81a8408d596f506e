"""Fused-collective microbenchmark on 2/4/8 GPUs.

    torchrun --nproc-per-node N bench_tp.py [--tokens 4096 16384 65536]

For every token count M and (K, N) shape, times on each rank with CUDA events
(max over ranks, L2 flushed between iterations by writing a 256 MB buffer):

* AG->GEMM  (column parallel, N sharded):  Y[M, N/t] = AG(x)[M, K] @ W[K, N/t]
    fused       our one-kernel all-gather + tcgen05 GEMM over NVLink peer memory
    nccl+ours   NCCL all_gather_into_tensor, then our tcgen05 GEMM
    nccl+cublas NCCL all_gather_into_tensor, then torch.matmul (the reference path)
* GEMM->RS  (row parallel, K sharded):  out[M/t, N] = RS(x[M, K/t] @ W[K/t, N])
    fused / nccl+ours / nccl+cublas likewise (NCCL reduce_scatter_tensor)

The roofline of a fused op is the slower of its FLOPs at the measured bf16
GEMM peak and the bytes it must move over NVLink at 770 GB/s per direction
(AG: (t-1)/t of the gathered input arrives; RS: (t-1)/t of the partial output
leaves). Prints one JSON line per (op, M, K, N).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
LINK_GBS = 770.0


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", type=int, nargs="+", default=[4096, 16384, 65536])
    p.add_argument("--shapes", default="4096x12288,4096x14336,14336x4096")
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    args = p.parse_args()
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(minutes=10), device_id=dev)
    rank, t = dist.get_rank(), dist.get_world_size()
    from nano_megatron_b200.ops import cuda as KC
    from nano_megatron_b200.ops import fused_tp
    from nano_megatron_b200.parallel import init_parallel
    pctx = init_parallel(tp_size=t)
    try:
        peak = json.load(open(os.path.join(HERE, "MEASURED_PEAKS.json")))["bf16_tflops"]
        peak_src = "bf16_tflops of measured"
    except (OSError, ValueError, KeyError):
        peak, peak_src = 1590.0, "fallback"
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        total = 0.0
        for _ in range(args.iters):
            flush.fill_(1)
            dist.barrier()
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            total += s.elapsed_time(e)
        ms = torch.tensor([total / args.iters], device=dev, dtype=torch.float64)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return ms.item()

    gen = torch.Generator(device=dev).manual_seed(rank)
    for shape in args.shapes.split(","):
        K, N = (int(v) for v in shape.split("x"))
        for M in args.tokens:
            # ---- all-gather -> GEMM (N sharded)
            x = torch.randn(M // t, K, device=dev, generator=gen).bfloat16()
            w = torch.randn(K, N // t, device=dev, generator=gen).bfloat16()
            gathered = torch.empty(M, K, device=dev, dtype=torch.bfloat16)

            def ag_nccl_ours():
                dist.all_gather_into_tensor(gathered, x)
                return KC.mm_nn(gathered, w)

            def ag_nccl_cublas():
                dist.all_gather_into_tensor(gathered, x)
                return gathered @ w

            res = {"fused": timed(lambda: fused_tp.all_gather_matmul(x, w, pctx)),
                   "nccl+ours": timed(ag_nccl_ours), "nccl+cublas": timed(ag_nccl_cublas)}
            fl = 2.0 * M * K * (N // t)
            comm = (t - 1) / t * M * K * 2
            roof = max(fl / (peak * 1e9), comm / (LINK_GBS * 1e6))
            if rank == 0:
                print(json.dumps({"op": "allgather_gemm", "tp": t, "M": M, "K": K, "N": N,
                                  "ms": {k: round(v, 4) for k, v in res.items()},
                                  "tflops_fused": round(fl / res["fused"] / 1e9, 1),
                                  "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / res["fused"], 3),
                                  "speedup_vs_nccl_cublas": round(res["nccl+cublas"] / res["fused"], 3),
                                  "peak": peak_src}), flush=True)
            del x, w, gathered
            # ---- GEMM -> reduce-scatter (K sharded)
            a = torch.randn(M, K // t, device=dev, generator=gen).bfloat16()
            w = torch.randn(K // t, N, device=dev, generator=gen).bfloat16()
            out = torch.empty(M // t, N, device=dev, dtype=torch.bfloat16)

            def rs_nccl_ours():
                dist.reduce_scatter_tensor(out, KC.mm_nn(a, w))
                return out

            def rs_nccl_cublas():
                dist.reduce_scatter_tensor(out, a @ w)
                return out

            res = {"fused": timed(lambda: fused_tp.matmul_reduce_scatter(a, w, pctx)),
                   "nccl+ours": timed(rs_nccl_ours), "nccl+cublas": timed(rs_nccl_cublas)}
            fl = 2.0 * M * (K // t) * N
            comm = (t - 1) / t * M * N * 2
            roof = max(fl / (peak * 1e9), comm / (LINK_GBS * 1e6))
            if rank == 0:
                print(json.dumps({"op": "gemm_reducescatter", "tp": t, "M": M, "K": K, "N": N,
                                  "ms": {k: round(v, 4) for k, v in res.items()},
                                  "tflops_fused": round(fl / res["fused"] / 1e9, 1),
                                  "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / res["fused"], 3),
                                  "speedup_vs_nccl_cublas": round(res["nccl+cublas"] / res["fused"], 3),
                                  "peak": peak_src}), flush=True)
            del a, w, out
            torch.cuda.empty_cache()
    KC.check_status(dev)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
