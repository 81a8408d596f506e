"""Resuming a run of the reference implementation in this package
(``import_reference_checkpoint``), against the reference itself (installed
under ``baseline/_ref``, or the directory named by ``NMB_REFERENCE_PATH``;
skipped when neither holds the ``nano_megatron`` package).

The reference trains two steps on a token file with its own model, AdamW,
1F1B, gradient finalization and clipping, and saves with its own
``save_checkpoint``. This package imports that directory into its model,
FusedAdamW and token stream, and both continue for two steps: the next batches,
the losses and the parameters must agree. A checkpoint written for another
configuration is refused before anything is loaded. The other direction:
``export_reference_checkpoint`` writes a directory the reference's own
``load_checkpoint`` resumes, and an export read back by the importer is exact.
"""

import os
import sys

import numpy as np
import pytest
import torch

REF = os.environ.get("NMB_REFERENCE_PATH") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")

KW = dict(vocab_size=64, n_layer=2, n_head=4, n_embd=32, seq_len=8)


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "nano_megatron")):
        pytest.skip(f"reference package not found under {REF}")
    sys.path.insert(0, REF)
    try:
        import nano_megatron.checkpoint as rckpt
        import nano_megatron.data as rdata
        import nano_megatron.grads as rgrads
        import nano_megatron.model as rmodel
        import nano_megatron.parallel as rpar
        import nano_megatron.pipeline as rpipe
        yield rmodel, rpipe, rgrads, rckpt, rdata, rpar
    finally:
        sys.path.remove(REF)


def _token_file(tmp_path):
    path = tmp_path / "tokens.bin"
    np.random.default_rng(0).integers(0, KW["vocab_size"], 5000, dtype=np.uint16).tofile(path)
    return path


def _ref_step(ref, model, opt, stream, cfg, ctx):
    rmodel, rpipe, rgrads, *_ = ref
    opt.zero_grad(set_to_none=True)
    batches = [stream.next_batch(2) for _ in range(2)]
    losses = rpipe.forward_backward_1f1b(model, batches, cfg, "cpu", ctx)
    rgrads.finalize_gradients(model, ctx, tie_embeddings=True)
    rgrads.clip_grad_norm(model, ctx, 1.0, tie_embeddings=True)
    opt.step()
    return torch.stack(losses).sum(), batches


def _our_step(model, opt, stream, cfg, ctx):
    from nano_megatron_b200 import forward_backward_1f1b
    from nano_megatron_b200.parallel.grads import clip_grad_norm, finalize_gradients
    opt.zero_grad()
    batches = [stream.next_batch(2) for _ in range(2)]
    losses = forward_backward_1f1b(model, batches, cfg, "cpu", ctx)
    finalize_gradients(model, ctx, tie_embeddings=True)
    clip_grad_norm(model, ctx, 1.0, tie_embeddings=True)
    opt.step()
    return torch.stack(losses).sum(), batches


def test_resume_a_reference_run(ref, tmp_path):
    rmodel, rpipe, rgrads, rckpt, rdata, rpar = ref
    from nano_megatron_b200 import GPT, GPTConfig, ParallelContext
    from nano_megatron_b200.optim import FusedAdamW
    from nano_megatron_b200.utils.checkpoint import import_reference_checkpoint
    from nano_megatron_b200.utils.data import TokenStream

    tokens = _token_file(tmp_path)
    rctx = rpar.ParallelContext.single()
    rcfg = rmodel.GPTConfig(**KW)
    torch.manual_seed(0)
    r = rmodel.GPT(rcfg)
    r_opt = torch.optim.AdamW(r.parameters(), lr=1e-3)
    r_stream = rdata.TokenStream(tokens, dtype="uint16", seq_len=KW["seq_len"])
    for _ in range(2):
        _ref_step(ref, r, r_opt, r_stream, rcfg, rctx)
    step_dir = tmp_path / "step_00000002"
    rckpt.save_checkpoint(step_dir, r, r_opt, rctx, step=2, data=r_stream, extra={"note": "ref"})

    cfg = GPTConfig(**KW)
    ctx = ParallelContext.single()
    torch.manual_seed(123)  # different init: everything must come from the checkpoint
    m = GPT(cfg, ctx)
    m_opt = FusedAdamW(m, lr=5e-2)
    m_stream = TokenStream(tokens, dtype="uint16", seq_len=KW["seq_len"])
    step, extra = import_reference_checkpoint(step_dir, m, m_opt, ctx, data=m_stream)
    assert step == 2 and extra == {"note": "ref"}
    assert m_opt.param_groups[0]["lr"] == 1e-3 and m_opt.step_count == 2
    for (n1, p1), (n2, p2) in zip(r.named_parameters(), m.named_parameters(), strict=True):
        assert n1 == n2 and torch.equal(p1, p2)

    for _ in range(2):
        lr_, br = _ref_step(ref, r, r_opt, r_stream, rcfg, rctx)
        lo, bo = _our_step(m, m_opt, m_stream, cfg, ctx)
        for (x1, y1), (x2, y2) in zip(br, bo, strict=True):
            assert torch.equal(x1, x2) and torch.equal(y1, y2)
        torch.testing.assert_close(lo, lr_, rtol=1e-5, atol=1e-6)
    for p1, p2 in zip(r.parameters(), m.parameters(), strict=True):
        torch.testing.assert_close(p2, p1, rtol=1e-4, atol=1e-6)


def test_refuses_a_checkpoint_of_another_configuration(ref, tmp_path):
    rmodel, rpipe, rgrads, rckpt, rdata, rpar = ref
    from nano_megatron_b200 import GPT, GPTConfig, ParallelContext
    from nano_megatron_b200.optim import FusedAdamW
    from nano_megatron_b200.utils.checkpoint import CheckpointError, import_reference_checkpoint

    rctx = rpar.ParallelContext.single()
    torch.manual_seed(0)
    r = rmodel.GPT(rmodel.GPTConfig(**KW))
    r_opt = torch.optim.AdamW(r.parameters(), lr=1e-3)
    rckpt.save_checkpoint(tmp_path / "s", r, r_opt, rctx, step=0)
    other = GPT(GPTConfig(**{**KW, "n_layer": 4}), ParallelContext.single())
    before = [p.detach().clone() for p in other.parameters()]
    with pytest.raises(CheckpointError, match="n_layer"):
        import_reference_checkpoint(tmp_path / "s", other, FusedAdamW(other), ParallelContext.single())
    assert all(torch.equal(a, p) for a, p in zip(before, other.parameters(), strict=True))
    theta = GPT(GPTConfig(**KW, rope_theta=500000.0), ParallelContext.single())
    with pytest.raises(CheckpointError, match="RoPE theta"):
        import_reference_checkpoint(tmp_path / "s", theta, FusedAdamW(theta), ParallelContext.single())


def test_reference_resumes_an_exported_checkpoint(ref, tmp_path):
    """The other direction: this package trains two steps and exports; the
    reference's own load_checkpoint resumes it, and both continue in lockstep."""
    rmodel, rpipe, rgrads, rckpt, rdata, rpar = ref
    from nano_megatron_b200 import GPT, GPTConfig, ParallelContext
    from nano_megatron_b200.optim import FusedAdamW
    from nano_megatron_b200.utils.checkpoint import export_reference_checkpoint
    from nano_megatron_b200.utils.data import TokenStream

    tokens = _token_file(tmp_path)
    cfg = GPTConfig(**KW)
    ctx = ParallelContext.single()
    torch.manual_seed(0)
    m = GPT(cfg, ctx)
    m_opt = FusedAdamW(m, lr=1e-3)
    m_stream = TokenStream(tokens, dtype="uint16", seq_len=KW["seq_len"])
    for _ in range(2):
        _our_step(m, m_opt, m_stream, cfg, ctx)
    step_dir = tmp_path / "step_00000002"
    export_reference_checkpoint(step_dir, m, m_opt, ctx, step=2, data=m_stream, extra={"note": "ours"})

    rctx = rpar.ParallelContext.single()
    rcfg = rmodel.GPTConfig(**KW)
    torch.manual_seed(123)  # different init: everything must come from the checkpoint
    r = rmodel.GPT(rcfg)
    r_opt = torch.optim.AdamW(r.parameters(), lr=5e-2)
    r_stream = rdata.TokenStream(tokens, dtype="uint16", seq_len=KW["seq_len"])
    step, extra = rckpt.load_checkpoint(step_dir, r, r_opt, rctx, data=r_stream)
    assert step == 2 and extra == {"note": "ours"}
    assert r_opt.param_groups[0]["lr"] == 1e-3
    for (n1, p1), (n2, p2) in zip(r.named_parameters(), m.named_parameters(), strict=True):
        assert n1 == n2 and torch.equal(p1, p2)

    for _ in range(2):
        lr_, br = _ref_step(ref, r, r_opt, r_stream, rcfg, rctx)
        lo, bo = _our_step(m, m_opt, m_stream, cfg, ctx)
        for (x1, y1), (x2, y2) in zip(br, bo, strict=True):
            assert torch.equal(x1, x2) and torch.equal(y1, y2)
        torch.testing.assert_close(lr_, lo, rtol=1e-5, atol=1e-6)
    for p1, p2 in zip(r.parameters(), m.parameters(), strict=True):
        torch.testing.assert_close(p1, p2, rtol=1e-4, atol=1e-6)


def test_export_then_import_is_exact(ref, tmp_path):
    from nano_megatron_b200 import GPT, GPTConfig, ParallelContext
    from nano_megatron_b200.optim import FusedAdamW
    from nano_megatron_b200.utils.checkpoint import export_reference_checkpoint, import_reference_checkpoint
    from nano_megatron_b200.utils.data import TokenStream

    tokens = _token_file(tmp_path)
    cfg, ctx = GPTConfig(**KW), ParallelContext.single()
    torch.manual_seed(0)
    a = GPT(cfg, ctx)
    a_opt = FusedAdamW(a, lr=2e-3, weight_decay=0.05)
    a_stream = TokenStream(tokens, dtype="uint16", seq_len=KW["seq_len"])
    for _ in range(3):
        _our_step(a, a_opt, a_stream, cfg, ctx)
    export_reference_checkpoint(tmp_path / "s", a, a_opt, ctx, step=3, data=a_stream)
    torch.manual_seed(9)
    b = GPT(cfg, ctx)
    b_opt = FusedAdamW(b)
    b_stream = TokenStream(tokens, dtype="uint16", seq_len=KW["seq_len"])
    assert import_reference_checkpoint(tmp_path / "s", b, b_opt, ctx, data=b_stream)[0] == 3
    assert all(torch.equal(p, q) for p, q in zip(a.parameters(), b.parameters(), strict=True))
    assert torch.equal(a_opt.exp_avg, b_opt.exp_avg) and torch.equal(a_opt.exp_avg_sq, b_opt.exp_avg_sq)
    assert b_opt.step_count == 3 and b_opt.param_groups == a_opt.param_groups
    assert b_stream.cursor == a_stream.cursor


def test_export_refuses_what_the_reference_cannot_describe(ref, tmp_path):
    from nano_megatron_b200 import GPT, GPTConfig, ParallelContext
    from nano_megatron_b200.optim import FusedAdamW
    from nano_megatron_b200.utils.checkpoint import CheckpointError, export_reference_checkpoint

    for extra_cfg, why in (({"ffn_hidden_size": 96}, "SwiGLU width"), ({"rope_theta": 500000.0}, "RoPE theta")):
        m = GPT(GPTConfig(**KW, **extra_cfg), ParallelContext.single())
        with pytest.raises(CheckpointError, match=why):
            export_reference_checkpoint(tmp_path / "s", m, FusedAdamW(m), ParallelContext.single(), step=0)
        assert not (tmp_path / "s").exists()
