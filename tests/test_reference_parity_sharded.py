"""Sharded parity with the reference implementation itself (installed under
``baseline/_ref``, or the directory named by ``NMB_REFERENCE_PATH``; skipped
when neither holds the ``nano_megatron`` package).

Every rank of a Gloo group builds the reference's stage model at a TP / PP /
DP layout with its own seed, loads that state into this package's stage model
(strict keys and shapes), runs both packages' 1F1B on the same synthetic
batches and finalizes the gradients with each package's own functions. The
losses, every local gradient shard and the logical clip norm must agree to
fp32 rounding: a user moving a sharded run from the reference to this package
gets the same numbers.
"""

import os
import sys
import tempfile
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REF = os.environ.get("NMB_REFERENCE_PATH") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
pytestmark = pytest.mark.distributed

TOL = dict(rtol=1e-4, atol=1e-6)


def _rank(rank, world, init_file, tp, pp, sp, tied, recompute, driver, ref_path, results):
    sys.path.insert(0, ref_path)
    import nano_megatron.grads as rgrads
    import nano_megatron.model as rmodel
    import nano_megatron.parallel as rpar
    import nano_megatron.pipeline as rpipe

    from nano_megatron_b200 import GPT, GPTConfig, forward_backward_1f1b, init_parallel
    from nano_megatron_b200.parallel.grads import clip_grad_norm, finalize_gradients
    from nano_megatron_b200.utils.data import synthetic_batches

    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    failures = []
    try:
        rctx = rpar.init_parallel(tp_size=tp, pp_size=pp)
        ctx = init_parallel(tp_size=tp, pp_size=pp)
        kw = dict(vocab_size=64, n_layer=2 * pp, n_head=4, n_embd=32, seq_len=8, sequence_parallel=sp,
                  tie_word_embeddings=tied, recompute=recompute)
        rcfg, cfg = rmodel.GPTConfig(**kw), GPTConfig(**kw)
        torch.manual_seed(1000 + rank)
        ref = rmodel.GPT(rcfg, rctx)
        ours = GPT(cfg, ctx)
        ours.load_state_dict(ref.state_dict(), strict=True)
        ref.train()
        ours.train()
        batches = synthetic_batches(cfg, 2, 4, 0, ctx.dp_rank)
        l_ref = rpipe.forward_backward_1f1b(ref, batches, rcfg, "cpu", rctx)
        if driver == "reference":  # the reference's own schedule drives this package's stage model
            l_ours = rpipe.forward_backward_1f1b(ours, batches, cfg, "cpu", rctx)
        else:
            l_ours = forward_backward_1f1b(ours, batches, cfg, "cpu", ctx)
        if ctx.is_last_stage:
            a, b = torch.stack(l_ours).sum(), torch.stack(l_ref).sum()
            if not torch.allclose(a, b, **TOL):
                failures.append(f"loss {a.item():.7f} != {b.item():.7f}")
        rgrads.finalize_gradients(ref, rctx, tie_embeddings=tied, sequence_parallel=sp)
        finalize_gradients(ours, ctx, tie_embeddings=tied, sequence_parallel=sp)
        ref_params = dict(ref.named_parameters())
        for name, p in ours.named_parameters():
            r = ref_params.get(name)
            if r is None or r.grad is None or p.grad is None:
                failures.append(f"{name}: missing gradient")
            elif not torch.allclose(p.grad, r.grad, **TOL):
                failures.append(f"{name}: max |diff| {(p.grad - r.grad).abs().max().item():.3e}")
        n_ref = rgrads.clip_grad_norm(ref, rctx, 1.0, tie_embeddings=tied)
        n_ours = clip_grad_norm(ours, ctx, 1.0, tie_embeddings=tied)
        if not torch.allclose(n_ours.double(), n_ref.double(), **TOL):
            failures.append(f"clip norm {n_ours.item():.7f} != {n_ref.item():.7f}")
    except Exception as e:  # reported to the parent as a failure of this rank
        failures.append(f"{type(e).__name__}: {e}")
    finally:
        results.put((rank, failures))
        dist.destroy_process_group()


def _run(tp, pp, dp, sp, tied=True, recompute=False, driver="ours"):
    world = tp * pp * dp
    spawn = mp.get_context("spawn")
    results = spawn.Queue()
    with tempfile.TemporaryDirectory() as tmp:
        init_file = os.path.join(tmp, "init")
        procs = [spawn.Process(target=_rank, args=(r, world, init_file, tp, pp, sp, tied, recompute, driver, REF,
                                                        results))
                 for r in range(world)]
        for p in procs:
            p.start()
        got, deadline = {}, time.monotonic() + 240
        while len(got) < world and time.monotonic() < deadline:
            try:
                rank, failures = results.get(timeout=1)
                got[rank] = failures
            except Exception:
                if any(p.exitcode not in (None, 0) for p in procs):
                    break
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
    assert len(got) == world, f"{world - len(got)} ranks did not report"
    bad = {r: f for r, f in got.items() if f}
    assert not bad, bad


@pytest.mark.parametrize("tp,pp,dp,sp", [(2, 1, 1, True), (2, 1, 1, False), (1, 2, 1, False), (2, 2, 1, True),
                                         (1, 1, 2, False), (4, 1, 1, True), (2, 2, 2, True)],
                         ids=["tp2-sp", "tp2", "pp2", "tp2xpp2-sp", "dp2", "tp4-sp", "tp2xpp2xdp2-sp"])
def test_sharded_parity_with_reference(tp, pp, dp, sp):
    if not os.path.isdir(os.path.join(REF, "nano_megatron")):
        pytest.skip(f"reference package not found under {REF}")
    _run(tp, pp, dp, sp)


def test_sharded_parity_untied_with_recompute():
    """Untied embeddings (no tied-group sum) and whole-block recompute, at TP2 x PP2 with SP."""
    if not os.path.isdir(os.path.join(REF, "nano_megatron")):
        pytest.skip(f"reference package not found under {REF}")
    _run(2, 2, 1, True, tied=False, recompute=True)


def test_the_reference_schedule_drives_this_package_stages():
    """Stage models exchange the reference's activation shapes, so the
    reference's forward_backward_1f1b runs this package's stages at TP2 x PP2
    with SP and gets the reference's losses, gradients and clip norm."""
    if not os.path.isdir(os.path.join(REF, "nano_megatron")):
        pytest.skip(f"reference package not found under {REF}")
    _run(2, 2, 1, True, driver="reference")
