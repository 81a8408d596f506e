"""Logical-model gradient clipping with the TP/PP collectives replaced by known
peer contributions (no process groups)."""

import contextlib

import pytest
import torch
import torch.nn as nn

from nano_megatron_b200.parallel import ParallelContext
from nano_megatron_b200.parallel import grads

TOL = dict(rtol=1e-6, atol=1e-6)


class _W(nn.Module):
    def __init__(self, g, sharded):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(len(g)))
        self.weight.grad = torch.tensor(g, dtype=torch.float32)
        self.weight.tensor_parallel_sharded = sharded


class _Stage(nn.Module):
    def __init__(self, pp_rank, tp_rank):
        super().__init__()
        shard = {(0, 0): [3.0], (0, 1): [4.0], (1, 0): [5.0], (1, 1): [12.0]}
        repl = {0: [2.0], 1: [6.0]}
        emb = {0: [1.0, 2.0], 1: [2.0, 1.0]}
        self.shard = _W(shard[pp_rank, tp_rank], True)
        self.replicated = _W(repl[pp_rank], False)
        if pp_rank == 0:
            self.embedding = _W(emb[tp_rank], True)
        else:
            self.lm_head = _W(emb[tp_rank], True)


@contextlib.contextmanager
def fake_groups(*, tp_size, pp_size, pp_rank, tp_peer=0.0, pp_peer=0.0):
    tp_group, pp_group, dp_group = object(), object(), object()
    calls = []
    ctx = ParallelContext(rank=pp_rank * tp_size, world_size=tp_size * pp_size * 2,
                          tp_size=tp_size, tp_rank=0, pp_size=pp_size, pp_rank=pp_rank,
                          dp_size=2, dp_rank=0, tp_group=tp_group, pp_group=pp_group,
                          dp_group=dp_group, tp_ranks=tuple(range(tp_size)),
                          pp_ranks=tuple(i * tp_size for i in range(pp_size)), dp_ranks=(0, tp_size))
    original = grads.dist.all_reduce

    def fake(tensor, group=None, **_):
        if group is tp_group:
            calls.append("tp")
            tensor.add_(tp_peer)
        elif group is pp_group:
            calls.append("pp")
            tensor.add_(pp_peer)
        elif group is dp_group:
            raise AssertionError("the gradient norm must never be reduced over DP")
        else:
            raise AssertionError("unexpected group")

    grads.dist.all_reduce = fake
    try:
        yield calls, ctx
    finally:
        grads.dist.all_reduce = original


def test_tp_pp_dp_tied_norm_and_scaling():
    local = {(0, 0): 16.0, (0, 1): 23.0, (1, 0): 43.0, (1, 1): 162.0}
    stage = {0: 39.0, 1: 205.0}
    expected = torch.tensor(244.0, dtype=torch.float64).sqrt()
    max_norm = expected.item() / 2
    scale = max_norm / (expected.item() + 1e-6)
    for pp_rank in (0, 1):
        for tp_rank in (0, 1):
            model = _Stage(pp_rank, tp_rank)
            before = {n: p.grad.clone() for n, p in model.named_parameters()}
            with fake_groups(tp_size=2, pp_size=2, pp_rank=pp_rank,
                             tp_peer=local[pp_rank, 1 - tp_rank], pp_peer=stage[1 - pp_rank]) as (calls, ctx):
                norm = grads.clip_grad_norm(model, ctx, max_norm, tie_embeddings=True)
            assert calls == ["tp", "pp"]
            torch.testing.assert_close(norm, expected, **TOL)
            for n, p in model.named_parameters():
                torch.testing.assert_close(p.grad, before[n] * scale, **TOL)


def test_tied_lm_head_counted_only_when_tied():
    model = nn.Module()
    model.lm_head = _W([3.0], True)
    with fake_groups(tp_size=1, pp_size=2, pp_rank=1, pp_peer=16.0) as (_, ctx):
        n = grads.clip_grad_norm(model, ctx, 100.0, tie_embeddings=False)
    torch.testing.assert_close(n, torch.tensor(5.0, dtype=torch.float64), **TOL)
    model.lm_head.weight.grad.fill_(3.0)
    with fake_groups(tp_size=1, pp_size=2, pp_rank=1, pp_peer=16.0) as (_, ctx):
        n = grads.clip_grad_norm(model, ctx, 100.0, tie_embeddings=True)
    torch.testing.assert_close(n, torch.tensor(4.0, dtype=torch.float64), **TOL)


def test_limits_and_empty_gradients():
    model = nn.Module()
    model.weight = nn.Parameter(torch.zeros(2))
    model.weight.grad = torch.tensor([3.0, 4.0])
    with fake_groups(tp_size=1, pp_size=1, pp_rank=0) as (_, ctx):
        assert grads.clip_grad_norm(model, ctx, 100.0).item() == 5.0
    assert torch.equal(model.weight.grad, torch.tensor([3.0, 4.0]))
    with fake_groups(tp_size=1, pp_size=1, pp_rank=0) as (_, ctx):
        assert grads.clip_grad_norm(model, ctx, 0.0).item() == 5.0
    assert torch.equal(model.weight.grad, torch.zeros(2))
    model.weight.grad = None
    with fake_groups(tp_size=1, pp_size=1, pp_rank=0) as (_, ctx):
        assert grads.clip_grad_norm(model, ctx, 1.0).item() == 0.0
    with pytest.raises(ValueError):
        grads.clip_grad_norm(model, ParallelContext.single(), -1.0)


def test_flat_buffer_model_clip_matches_torch():
    from nano_megatron_b200.models import GPT, GPTConfig
    torch.manual_seed(0)
    model = GPT(GPTConfig(vocab_size=32, n_layer=2, n_head=2, n_embd=16, seq_len=4))
    model(torch.randint(0, 32, (2, 4)), torch.randint(0, 32, (2, 4))).backward()
    grads_copy = [p.grad.clone() for p in model.parameters()]
    ref = nn.ParameterList([nn.Parameter(torch.zeros_like(g)) for g in grads_copy])
    for p, g in zip(ref, grads_copy):
        p.grad = g.clone()
    expected = torch.nn.utils.clip_grad_norm_(ref.parameters(), 0.01)
    norm = grads.clip_grad_norm(model, ParallelContext.single(), 0.01)
    torch.testing.assert_close(norm.float(), expected.float(), rtol=1e-5, atol=1e-7)
    for p, r in zip(model.parameters(), ref.parameters()):
        torch.testing.assert_close(p.grad, r.grad, rtol=1e-5, atol=1e-8)
