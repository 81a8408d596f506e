"""The reference's public modules and functions, called the way the reference
calls them, give the same values and gradients in this package (the reference
is installed under ``baseline/_ref``, or the directory named by
``NMB_REFERENCE_PATH``; skipped when neither holds the ``nano_megatron``
package).

Each case builds the reference's module, copies its state into this package's
module of the same name and runs both on the same batch-first inputs; the
outputs, the input gradients and every parameter gradient must agree to fp32
rounding. This runs in one process at TP=1, on Gloo ranks at TP=2 with and
without sequence parallelism, and at TP=4 with it. Covered: ``ColumnParallelLinear``,
``RowParallelLinear``, ``VocabParallelEmbedding``, ``RMSNorm``,
``ParallelAttention``, ``ParallelMLP``, ``TransformerLayer``,
``ParallelLMHead``, ``vocab_parallel_cross_entropy`` and the four
tensor/sequence-parallel mappings.
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
TOL = dict(rtol=1e-4, atol=1e-6)
B, S, H, HEADS, V = 2, 8, 32, 4, 64


def _have_reference() -> bool:
    return os.path.isdir(os.path.join(REF, "nano_megatron"))


def _import_reference():
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import nano_megatron.cross_entropy as rce
    import nano_megatron.mappings as rmap
    import nano_megatron.model as rmodel
    import nano_megatron.parallel as rpar
    import nano_megatron.tp_layers as rtp
    return rmodel, rtp, rmap, rce, rpar


def _randn(seed, *shape):
    return torch.randn(tuple(shape), generator=torch.Generator().manual_seed(seed))


def _compare(name, ref_mod, our_mod, call, inputs, failures, seed=7):
    """Run ``call(module, *inputs)`` on both modules (our module holding the
    reference's state); compare outputs, input gradients and parameter gradients."""
    if ref_mod is not None:
        our_mod.load_state_dict(ref_mod.state_dict(), strict=True)
    xr = [t.clone().requires_grad_(t.is_floating_point()) for t in inputs]
    xo = [t.clone().requires_grad_(t.is_floating_point()) for t in inputs]
    yr, yo = call(ref_mod, *xr, ours=False), call(our_mod, *xo, ours=True)
    if yr.shape != yo.shape:
        failures.append(f"{name}: shape {tuple(yo.shape)} != reference {tuple(yr.shape)}")
        return
    if not torch.allclose(yo.float(), yr.float(), **TOL):
        failures.append(f"{name}: output max |diff| {(yo.float() - yr.float()).abs().max().item():.3e}")
    g = _randn(seed, *yr.shape)
    (yr.float() * g).sum().backward()
    (yo.float() * g).sum().backward()
    for i, (a, b) in enumerate(zip(xr, xo)):
        if a.requires_grad and not torch.allclose(b.grad, a.grad, **TOL):
            failures.append(f"{name}: input {i} gradient max |diff| {(b.grad - a.grad).abs().max().item():.3e}")
    if ref_mod is None:
        return
    ours = dict(our_mod.named_parameters())
    for pname, p in ref_mod.named_parameters():
        q = ours[pname]
        if p.grad is None or q.grad is None:
            if (p.grad is None) != (q.grad is None):
                failures.append(f"{name}.{pname}: gradient present in only one package")
        elif not torch.allclose(q.grad, p.grad, **TOL):
            failures.append(f"{name}.{pname}: gradient max |diff| {(q.grad - p.grad).abs().max().item():.3e}")


def _check_all(rctx, ctx, sp, failures):
    """Every case at this rank; ``rctx``/``ctx`` are the two packages' contexts."""
    rmodel, rtp, rmap, rce, _ = _import_reference()
    import nano_megatron_b200.models as M
    import nano_megatron_b200.parallel as P

    tp, rank = ctx.tp_size, ctx.tp_rank
    s_local = S // tp if sp else S
    x_full = _randn(1, B, S, H)
    x_in = x_full.chunk(tp, dim=1)[rank].contiguous() if sp else x_full
    kw = dict(vocab_size=V, n_layer=1, n_head=HEADS, n_embd=H, seq_len=S, sequence_parallel=sp)
    rcfg, cfg = rmodel.GPTConfig(**kw), M.GPTConfig(**kw)
    cos, sin = rmodel.build_rope_cache(S, H // HEADS, torch.device("cpu"))

    def build(ref_factory, our_factory):
        torch.manual_seed(100 + rank)
        r = ref_factory()
        return r, our_factory()

    for flag in (True, False):
        r, o = build(lambda: rtp.ColumnParallelLinear(H, 2 * H, rctx),
                     lambda: M.ColumnParallelLinear(H, 2 * H, ctx))
        with torch.no_grad():
            r.bias.normal_()
        _compare(f"ColumnParallelLinear(reduce_input_grad={flag})", r, o,
                 lambda m, x, ours: m(x, reduce_input_grad=flag), [x_full], failures)

    r, o = build(lambda: rtp.RowParallelLinear(2 * H, H, rctx), lambda: M.RowParallelLinear(2 * H, H, ctx))
    with torch.no_grad():
        r.bias.normal_()
    _compare("RowParallelLinear", r, o, lambda m, x, ours: m(x, sequence_parallel=sp),
             [_randn(10 + rank, B, S, 2 * H // tp)], failures)

    ids = torch.randint(0, V, (B, S), generator=torch.Generator().manual_seed(3))
    r, o = build(lambda: rtp.VocabParallelEmbedding(V, H, rctx), lambda: M.VocabParallelEmbedding(V, H, ctx))
    _compare("VocabParallelEmbedding", r, o, lambda m, i, ours: m(i, sequence_parallel=sp), [ids], failures)

    r, o = build(lambda: rmodel.RMSNorm(H), lambda: M.RMSNorm(H))
    with torch.no_grad():
        r.weight.normal_()
    _compare("RMSNorm", r, o, lambda m, x, ours: m(x), [x_in], failures)

    r, o = build(lambda: rmodel.ParallelAttention(rcfg, rctx), lambda: M.ParallelAttention(cfg, ctx))
    _compare("ParallelAttention", r, o, lambda m, x, ours: m(x, cos, sin), [x_in], failures)

    r, o = build(lambda: rmodel.ParallelMLP(rcfg, rctx), lambda: M.ParallelMLP(cfg, ctx))
    _compare("ParallelMLP", r, o, lambda m, x, ours: m(x), [x_in], failures)

    r, o = build(lambda: rmodel.TransformerLayer(rcfg, rctx), lambda: M.TransformerLayer(cfg, ctx))
    _compare("TransformerLayer", r, o, lambda m, x, ours: m(x, cos, sin), [x_in], failures)

    r, o = build(lambda: rmodel.ParallelLMHead(rcfg, rctx), lambda: M.ParallelLMHead(cfg, ctx))
    _compare("ParallelLMHead", r, o, lambda m, x, ours: m(x), [x_in], failures)

    per = V // tp
    start, end = rank * per, (rank + 1) * per
    target = torch.randint(0, V, (B, S), generator=torch.Generator().manual_seed(4))

    def ce(_m, logits, ours):
        fn, c = (M.vocab_parallel_cross_entropy, ctx) if ours else (rce.vocab_parallel_cross_entropy, rctx)
        return fn(logits, target, start, end, c)

    _compare("vocab_parallel_cross_entropy", None, None, ce, [_randn(20 + rank, B, S, per)], failures)

    mappings = [("copy_to_tensor_parallel_region", x_full),
                ("reduce_from_tensor_parallel_region", _randn(30 + rank, B, S, H)),
                ("gather_from_sequence_parallel_region", _randn(40 + rank, B, S // tp, H)),
                ("reduce_scatter_to_sequence_parallel_region", _randn(50 + rank, B, S, H))]
    for fname, x in mappings:
        def call(_m, t, ours, fname=fname):
            return getattr(P, fname)(t, ctx) if ours else getattr(rmap, fname)(t, rctx)
        _compare(fname, None, None, call, [x], failures)
    assert s_local > 0


def test_reference_modules_single_process():
    if not _have_reference():
        pytest.skip(f"reference package not found under {REF}")
    from nano_megatron_b200.parallel import ParallelContext
    rpar = _import_reference()[4]
    failures = []
    _check_all(rpar.ParallelContext.single(), ParallelContext.single(), False, failures)
    assert not failures, failures


def test_reference_autocast_call_matches_bf16_compute():
    """A layer called under the reference's bf16 autocast computes in bf16 here too."""
    if not _have_reference():
        pytest.skip(f"reference package not found under {REF}")
    rmodel = _import_reference()[0]
    import nano_megatron_b200.models as M
    from nano_megatron_b200.parallel import ParallelContext
    rpar = _import_reference()[4]
    kw = dict(vocab_size=V, n_layer=1, n_head=HEADS, n_embd=H, seq_len=S)
    torch.manual_seed(0)
    r = rmodel.TransformerLayer(rmodel.GPTConfig(**kw), rpar.ParallelContext.single())
    o = M.TransformerLayer(M.GPTConfig(**kw), ParallelContext.single())
    o.load_state_dict(r.state_dict())
    cos, sin = rmodel.build_rope_cache(S, H // HEADS, torch.device("cpu"))
    x = _randn(1, B, S, H).to(torch.bfloat16)
    with torch.autocast("cpu", dtype=torch.bfloat16):
        yr, yo = r(x, cos, sin), o(x, cos, sin)
    assert yo.dtype == yr.dtype == torch.bfloat16
    err = (yo.float() - yr.float()).norm() / yr.float().norm()
    assert err < 2e-2, err


def _rank(rank, world, init_file, sp, ref_path, results):
    os.environ["NMB_REFERENCE_PATH"] = ref_path
    failures = []
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        rpar = _import_reference()[4]
        from nano_megatron_b200.parallel import init_parallel
        rctx = rpar.init_parallel(tp_size=world)
        ctx = init_parallel(tp_size=world)
        _check_all(rctx, ctx, sp, failures)
    except Exception as e:  # reported to the parent as a failure of this rank
        failures.append(f"{type(e).__name__}: {e}")
    finally:
        results.put((rank, failures))
        dist.destroy_process_group()


@pytest.mark.distributed
@pytest.mark.parametrize("world,sp", [(2, False), (2, True), (4, True)], ids=["tp2", "tp2-sp", "tp4-sp"])
def test_reference_modules_tp(world, sp):
    if not _have_reference():
        pytest.skip(f"reference package not found under {REF}")
    spawn = mp.get_context("spawn")
    results = spawn.Queue()
    with tempfile.TemporaryDirectory() as tmp:
        init_file = os.path.join(tmp, "init")
        procs = [spawn.Process(target=_rank, args=(r, world, init_file, sp, REF, results))
                 for r in range(world)]
        for p in procs:
            p.start()
        got, deadline = {}, time.monotonic() + 180
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
