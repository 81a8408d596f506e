"""Tensor-parallel algebra on simulated ranks (no process groups).

Partial per-rank results are combined by the test itself, which proves that
column/row sharding reconstructs the full matmuls and vocab sharding
reconstructs cross entropy. Collectives are stubbed where a layer would issue
one.
"""

import torch
import torch.nn.functional as F

from nano_megatron_b200.models import ColumnParallelLinear, RowParallelLinear
from nano_megatron_b200.models.functional import WeightRef, lm_head_cross_entropy
from nano_megatron_b200.parallel import ParallelContext, mappings

TOL = dict(rtol=1e-5, atol=1e-6)


def simulated(tp, r):
    return ParallelContext(rank=r, world_size=tp, tp_size=tp, tp_rank=r, pp_size=1, pp_rank=0,
                           dp_size=1, dp_rank=0, tp_ranks=tuple(range(tp)), pp_ranks=(r,),
                           dp_ranks=(r,))


def test_column_row_pair_reconstructs_mlp():
    torch.manual_seed(0)
    x = torch.randn(3, 16)
    A, B = torch.randn(16, 32) * 0.1, torch.randn(32, 16) * 0.1
    expected = F.silu(x @ A) @ B
    for tp in (2, 4):
        total = torch.zeros(3, 16)
        for r in range(tp):
            ctx = simulated(tp, r)
            col = ColumnParallelLinear(16, 32, ctx, bias=False)
            row = RowParallelLinear(32, 16, ctx, bias=False)
            col.weight.data.copy_(torch.chunk(A, tp, dim=1)[r])
            row.weight.data.copy_(torch.chunk(B, tp, dim=0)[r])
            total += row(F.silu(col(x, reduce_input_grad=False)), reduce_output=False)
        torch.testing.assert_close(total, expected, **TOL)


def test_column_shard_gradients_concatenate():
    torch.manual_seed(0)
    x = torch.randn(3, 16)
    A = (torch.randn(16, 32) * 0.1).requires_grad_(True)
    (x @ A).pow(2).sum().backward()
    shards = []
    for r in range(4):
        col = ColumnParallelLinear(16, 32, simulated(4, r), bias=False)
        col.weight.data.copy_(torch.chunk(A.detach(), 4, dim=1)[r])
        col(x, reduce_input_grad=False).pow(2).sum().backward()
        shards.append(col.weight.grad)
    torch.testing.assert_close(torch.cat(shards, dim=1), A.grad, **TOL)


def test_row_shard_gradients_concatenate():
    torch.manual_seed(1)
    x = torch.randn(5, 32)
    B = (torch.randn(32, 8) * 0.1).requires_grad_(True)
    (x @ B).sin().sum().backward()
    for tp in (2, 4):
        shards = []
        for r in range(tp):
            row = RowParallelLinear(32, 8, simulated(tp, r), bias=False)
            row.weight.data.copy_(torch.chunk(B.detach(), tp, dim=0)[r])
            xr = torch.chunk(x, tp, dim=1)[r]
            # the upstream gradient of a row layer is the full output gradient
            y = xr @ B.detach()[r * 32 // tp:(r + 1) * 32 // tp]
            full = x @ B.detach()
            g = full.cos()
            out = row(xr, reduce_output=False)
            out.backward(g)
            shards.append(row.weight.grad)
        torch.testing.assert_close(torch.cat(shards, dim=0), B.grad, **TOL)


def test_vocab_parallel_cross_entropy_and_gradient():
    """LM head + CE on vocab shards, with the stats merge done by the test."""
    from nano_megatron_b200.ops import reference as ref
    torch.manual_seed(0)
    T, H, V = 10, 8, 16
    x = torch.randn(T, H)
    W = torch.randn(V, H)
    labels = torch.randint(0, V, (T,))
    logits = x @ W.t()
    expected = F.cross_entropy(logits, labels)
    for tp in (2, 4):
        per = V // tp
        mx, se, tl = [], [], []
        for r in range(tp):
            m, s, t, _ = ref.ce_local_stats(logits[:, r * per:(r + 1) * per], labels, r * per, (r + 1) * per)
            mx.append(m), se.append(s), tl.append(t)
        gm = torch.stack(mx).max(0).values
        gs = sum(s * (m - gm).exp() for s, m in zip(se, mx))
        loss = (gs.log() + gm - sum(tl)).mean()
        torch.testing.assert_close(loss, expected, **TOL)
    # tp=1 fused function: loss and gradients against autograd
    xr = x.clone().requires_grad_(True)
    Wr = W.clone().requires_grad_(True)
    F.cross_entropy(xr @ Wr.t(), labels).backward()
    xp = x.clone().requires_grad_(True)
    Wp = torch.nn.Parameter(W.clone())
    loss = lm_head_cross_entropy(xp, labels, WeightRef.of(Wp), ParallelContext.single(), "f",
                                 torch.float32, 0, V)
    loss.backward()
    torch.testing.assert_close(loss, expected, **TOL)
    torch.testing.assert_close(xp.grad, xr.grad, rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(Wp.grad, Wr.grad, rtol=1e-4, atol=1e-6)


def test_public_vocab_parallel_cross_entropy_matches_torch():
    from nano_megatron_b200.models.cross_entropy import vocab_parallel_cross_entropy
    torch.manual_seed(0)
    logits = torch.randn(2, 5, 16)
    labels = torch.randint(0, 16, (2, 5))
    a = logits.clone().requires_grad_(True)
    F.cross_entropy(a.view(-1, 16), labels.view(-1)).backward()
    b = logits.clone().requires_grad_(True)
    vocab_parallel_cross_entropy(b, labels, 0, 16, ParallelContext.single()).backward()
    torch.testing.assert_close(b.grad, a.grad, rtol=1e-4, atol=1e-6)


def test_f_and_g_compose_to_identity_with_stubbed_collectives(monkeypatch):
    ctx = simulated(2, 0)
    monkeypatch.setattr(mappings, "_all_reduce", lambda t, _g, _n: t)
    x = torch.randn(4, 8, requires_grad=True)
    y = mappings.reduce_from_tensor_parallel_region(mappings.copy_to_tensor_parallel_region(x, ctx), ctx)
    assert torch.equal(y, x)
    y.sum().backward()
    assert torch.equal(x.grad, torch.ones_like(x))
