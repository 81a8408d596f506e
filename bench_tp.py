"""Fused-collective microbenchmark (the fused-collective configuration of the target) on 2/4/8 GPUs.

    torchrun --nproc-per-node N bench_tp.py [--tokens 4096 16384 65536]

For every token count M and (K, N) shape, times on each rank with CUDA events
(max over ranks, L2 flushed between iterations by writing a 256 MB buffer):

* AG->GEMM  (column parallel, N sharded):  Y[M, N/t] = AG(x)[M, K] @ W[K, N/t]
    fused       our one-kernel all-gather + tcgen05 GEMM over NVLink peer memory
    nccl+ours   NCCL all_gather_into_tensor, then our tcgen05 GEMM
    nccl+cublas NCCL all_gather_into_tensor, then torch.matmul (the reference path)
* GEMM->RS  (row parallel, K sharded):  out[M/t, N] = RS(x[M, K/t] @ W[K/t, N])
    fused / nccl+ours / nccl+cublas likewise (NCCL reduce_scatter_tensor)

* LM head + vocab-parallel cross entropy (hidden 4096, vocab 128256, 16384
  tokens, uniform targets; ``--ce-tokens``/``--ce-hidden``/``--ce-vocab``):
    fused       forward: our all-gather -> GEMM with the CE-statistics epilogue
                and the symmetric-memory merge; backward: in-place
                softmax-minus-onehot, fused dgrad GEMM -> reduce-scatter, wgrad
    nccl+cublas the reference's path: NCCL all-gather, torch.matmul logits,
                fp32 softmax statistics with three NCCL all-reduces (MAX, SUM,
                SUM), backward in torch with an NCCL reduce-scatter

* Data-parallel gradient average of one fp32 bucket (``--ops dp``, 64 and 256 MB):
    ours        the two-shot NVLink kernel of csrc/dp_reduce.cu (1/dp applied in the pass)
    nccl        NCCL all_reduce with ReduceOp.AVG
  roofline: every rank receives (t-1)/t of the bucket and sends as much.

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


def bench_ce(args, pctx, dev, rank, t, timed, peak, peak_src):
    from nano_megatron_b200.ops import cuda as KC
    from nano_megatron_b200.ops import fused_tp
    M, H, V = args.ce_tokens, args.ce_hidden, args.ce_vocab
    vl = V // t
    vs, ve = rank * vl, (rank + 1) * vl
    g = torch.Generator(device=dev).manual_seed(1000)  # same labels on every rank
    labels = torch.randint(0, V, (M,), generator=g, device=dev)
    gr = torch.Generator(device=dev).manual_seed(2000 + rank)
    x = torch.randn(M // t, H, device=dev, generator=gr).bfloat16()
    w = (torch.randn(vl, H, device=dev, generator=gr) * 0.02).bfloat16()
    wgrad = torch.zeros(vl, H, device=dev)
    state = {}

    def fused_fwd():
        state["f"] = fused_tp.lm_head_cross_entropy(x, w, labels, vs, ve, pctx, gather=True)
        return state["f"][0]

    def fused_bwd():
        loss, logits, gm, gs, X = state["f"]
        d = KC.lm_head_ce_grad(X, w, labels, vs, (logits, gm, gs), torch.tensor(1.0 / M, device=dev),
                               inplace=True)
        dx = fused_tp.matmul_reduce_scatter(d, w, pctx, transpose_b=False)
        KC.mm_tn_acc(d, X, wgrad)
        return dx

    gathered = torch.empty(M, H, device=dev, dtype=torch.bfloat16)
    local = labels - vs
    owned = (local >= 0) & (local < vl)
    lidx = local.clamp(0, vl - 1)[:, None]

    def ref_fwd():
        # nano_megatron/cross_entropy.py:16-49 with the NCCL all-gather in front
        dist.all_gather_into_tensor(gathered, x)
        logits = (gathered @ w.t()).float()
        mx = logits.max(dim=-1).values
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        logits.sub_(mx[:, None])
        tl = torch.where(owned, logits.gather(1, lidx)[:, 0], torch.zeros_like(mx))
        dist.all_reduce(tl)
        logits.exp_()
        se = logits.sum(dim=-1)
        dist.all_reduce(se)
        logits.div_(se[:, None])
        state["r"] = logits
        return (se.log() - tl).mean()

    out = torch.empty(M // t, H, device=dev, dtype=torch.bfloat16)

    def ref_bwd():
        sm = state["r"]
        sm[owned, local[owned]] -= 1.0
        d = (sm * (1.0 / M)).bfloat16()
        dist.reduce_scatter_tensor(out, d @ w)
        wgrad.add_((d.t() @ gathered).float())
        return out

    # backward = (forward + backward) - forward: the backward consumes the forward's state
    res = {"fused_fwd": timed(fused_fwd)}
    res["fused_bwd"] = timed(lambda: (fused_fwd(), fused_bwd())) - res["fused_fwd"]
    res["ref_fwd"] = timed(ref_fwd)
    res["ref_bwd"] = timed(lambda: (ref_fwd(), ref_bwd())) - res["ref_fwd"]
    fl = 2.0 * M * H * vl
    comm = (t - 1) / t * M * H * 2
    roof_f = max(fl / (peak * 1e9), comm / (LINK_GBS * 1e6))
    roof_b = max(2 * fl / (peak * 1e9), comm / (LINK_GBS * 1e6))
    if rank == 0:
        print(json.dumps({"op": "lmhead_ce", "tp": t, "M": M, "H": H, "V": V,
                          "ms": {k: round(v, 4) for k, v in res.items()},
                          "roofline_ms": {"fwd": round(roof_f, 4), "bwd": round(roof_b, 4)},
                          "frac_of_roofline": {"fwd": round(roof_f / res["fused_fwd"], 3),
                                               "bwd": round(roof_b / res["fused_bwd"], 3)},
                          "speedup_vs_reference_path": {
                              "fwd": round(res["ref_fwd"] / res["fused_fwd"], 3),
                              "bwd": round(res["ref_bwd"] / res["fused_bwd"], 3)},
                          "peak": peak_src}), flush=True)
    del state, gathered
    torch.cuda.empty_cache()


def bench_dp(dev, rank, t, timed):
    from nano_megatron_b200.ops import dp_reduce
    from nano_megatron_b200.parallel import init_parallel
    ctx = init_parallel(tp_size=1, pp_size=1)  # all ranks form the DP group
    for mb in (64, 256):
        n = mb * (1 << 20) // 4

        class _Flat:  # the two members the workspace uses
            numel = n
            grad = torch.randn(n, device=dev)

            @classmethod
            def rehome_grad(cls, g):
                g.copy_(cls.grad)
                cls.grad = g

        ws = dp_reduce.DPWorkspace(ctx, _Flat)
        plain = torch.randn(n, device=dev)
        res = {"ours": timed(lambda: ws.all_reduce_avg(0, n)),
               "nccl": timed(lambda: dist.all_reduce(plain, op=dist.ReduceOp.AVG))}
        roof = (t - 1) / t * n * 4 / (LINK_GBS * 1e6)
        if rank == 0:
            print(json.dumps({"op": "dp_allreduce_avg", "ranks": t, "MB": mb,
                              "ms": {k: round(v, 4) for k, v in res.items()},
                              "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / res["ours"], 3),
                              "speedup_vs_nccl": round(res["nccl"] / res["ours"], 3)}), flush=True)
        del ws, plain
        torch.cuda.empty_cache()


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", type=int, nargs="+", default=[4096, 16384, 65536])
    p.add_argument("--shapes", default="4096x12288,4096x14336,14336x4096")
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--ops", default="ag,rs,ce", help="comma list of ag, rs, ce, dp")
    p.add_argument("--ce-tokens", type=int, default=16384)
    p.add_argument("--ce-hidden", type=int, default=4096)
    p.add_argument("--ce-vocab", type=int, default=128256)
    args = p.parse_args()
    ops = set(args.ops.split(","))
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
    if "ce" in ops:
        bench_ce(args, pctx, dev, rank, t, timed, peak, peak_src)
    if "dp" in ops:
        bench_dp(dev, rank, t, timed)
    for shape in args.shapes.split(","):
        K, N = (int(v) for v in shape.split("x"))
        for M in args.tokens:
            if "ag" not in ops:
                break
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
        for M in args.tokens:
            if "rs" not in ops:
                break
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
