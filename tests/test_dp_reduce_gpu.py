"""Data-parallel averaging kernel (NVLink peer memory) on 2, 4 or 8 GPUs (every
size the box has) against the plain average, span by span, bitwise repeatable;
the averaged gradients of a data-parallel training step with it against the
NCCL path; and, with 4 or more GPUs, a TP=2 sequence-parallel x DP step whose
buckets run on the communication stream beside the fused TP kernels of the
backward. Needs at least 2 GPUs (skipped otherwise)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:  # pragma: no cover
    pytest.skip("needs 2 CUDA GPUs", allow_module_level=True)

WORLDS = [w for w in (2, 4, 8) if w <= torch.cuda.device_count()]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    failures = []
    try:
        from nano_megatron_b200.ops import cuda as KC
        from nano_megatron_b200.ops import dp_reduce
        from nano_megatron_b200.parallel import init_parallel
        dp_reduce.TIMEOUT_S = 10.0
        ctx = init_parallel(tp_size=1, pp_size=1)  # every rank in one DP group

        class _Flat:  # the two members DPWorkspace uses
            def __init__(self, n):
                self.numel = n
                self.grad = torch.zeros(n, device=dev)

            def rehome_grad(self, g):
                g.copy_(self.grad)
                self.grad = g

        n = (1 << 22) + 64
        flat = _Flat(n)
        ws = dp_reduce.DPWorkspace(ctx, flat)
        for it in range(3):
            gen = torch.Generator(device=dev).manual_seed(100 * it + rank)
            flat.grad.copy_(torch.randn(n, generator=gen, device=dev))
            parts = [torch.empty_like(flat.grad) for _ in range(world)]
            dist.all_gather(parts, flat.grad)
            want = sum(parts) / world
            before = flat.grad.clone()
            spans = [(0, 4096), (4096, 4096 + 262144), (4096 + 262144, n - 64), (n - 64, n)]
            for start, end in spans:
                ws.all_reduce_avg(start, end)
            torch.cuda.synchronize()
            err = (flat.grad - want).abs().max().item()
            if err > 1e-6:
                failures.append(f"iteration {it}: max error {err}")
            first = flat.grad.clone()
            flat.grad.copy_(before)
            dist.barrier()
            for start, end in spans:
                ws.all_reduce_avg(start, end)
            torch.cuda.synchronize()
            if not torch.equal(flat.grad, first):
                failures.append(f"iteration {it}: not bitwise repeatable")
        KC.check_status(dev)

        # DP=2 training step: bucketed NVLink averaging vs one NCCL average after backward
        from nano_megatron_b200 import GPTConfig
        from nano_megatron_b200.train import Trainer
        cfg = GPTConfig(vocab_size=1024, n_layer=2, n_head=4, n_embd=512, seq_len=256, ffn_hidden_size=1024,
                        compute_dtype="bfloat16", tie_word_embeddings=False, init_std=0.05)
        gen = torch.Generator().manual_seed(7 + rank)
        batches = [(torch.randint(0, 1024, (1, 256), generator=gen), torch.randint(0, 1024, (1, 256), generator=gen))
                   for _ in range(3)]
        params = {}
        for mb in (0.0, 0.25):
            trainer = Trainer(cfg, ctx, dev, lr=1e-3, seed=3, init_device=dev, dp_bucket_mb=mb)
            trainer.train_step(batches)
            torch.cuda.synchronize()
            params[mb] = trainer.model.flat_buffers.grad.clone()  # the DP-averaged gradients
            if mb > 0 and trainer.bucketer is None:
                failures.append("bucketer not created")
        diff = ((params[0.0] - params[0.25]).norm() / params[0.0].norm()).item()
        if diff > 1e-5:
            failures.append(f"trainer step: bucketed NVLink vs NCCL gradient difference {diff}")
        KC.check_status(dev)

        if world >= 4:
            # TP=2 (fused kernels in backward) x DP: buckets on the comm stream
            from nano_megatron_b200.ops import fused_tp
            fused_tp.TIMEOUT_S = 10.0
            tctx = init_parallel(tp_size=2, pp_size=1)
            cfg = GPTConfig(vocab_size=1024, n_layer=2, n_head=4, n_embd=512, seq_len=512,
                            ffn_hidden_size=1024, compute_dtype="bfloat16", tie_word_embeddings=False,
                            sequence_parallel=True, init_std=0.05)
            gen = torch.Generator().manual_seed(70 + tctx.dp_rank)
            batches = [(torch.randint(0, 1024, (1, 512), generator=gen),
                        torch.randint(0, 1024, (1, 512), generator=gen)) for _ in range(3)]
            grads = {}
            for mb in (0.0, 0.25):
                trainer = Trainer(cfg, tctx, dev, lr=1e-3, seed=3, init_device=dev, dp_bucket_mb=mb)
                trainer.train_step(batches)
                torch.cuda.synchronize()
                grads[mb] = trainer.model.flat_buffers.grad.clone()
                if mb > 0:
                    stats = trainer.bucketer.last_step
                    if not stats["on_comm_stream"] or stats["during_backward"] < 2:
                        failures.append(f"TPxDP buckets did not overlap backward: {stats}")
            diff = ((grads[0.0] - grads[0.25]).norm() / grads[0.0].norm()).item()
            if diff > 1e-5:
                failures.append(f"TPxDP step: bucketed vs one average gradient difference {diff}")
            KC.check_status(dev)
    except Exception as exc:  # report instead of hanging the peer
        failures.append(f"exception: {exc!r}")
    q.put((rank, failures))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", WORLDS)
def test_dp_allreduce(world):
    from tests.test_fused_tp_gpu import run_ranks
    results = run_ranks(_worker, world)
    assert all(results.get(r) == [] for r in range(world)), results
