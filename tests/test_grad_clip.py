"""Logical-model gradient clipping without sockets.

Each virtual rank of a TP x PP grid runs ``clip_grad_norm`` in its own thread.
The process groups are in-process objects: ``all_reduce`` over a group is a
barrier exchange among that group's threads, so the collectives run for real
(order, membership, values) without ``torch.distributed``. The data-parallel
group refuses every call, because the norm of DP replicas must never be
reduced over DP. The expected norm comes from the unsharded logical model.
"""

import threading
from contextlib import contextmanager

import pytest
import torch
import torch.nn as nn

from nano_megatron_b200.parallel import ParallelContext, grads


class _Group:
    def __init__(self, kind, members):
        self.kind, self.members = kind, tuple(members)
        self.barrier = threading.Barrier(len(members))
        self.slots = {}


class ThreadWorld:
    """Virtual ranks ``(pp, tp)`` of DP lane 0 in a world with ``dp`` lanes."""

    def __init__(self, tp, pp, dp=2):
        self.tp, self.pp, self.dp = tp, pp, dp
        self.local = threading.local()
        self.log, self.dp_calls = [], []
        self.tp_groups = {p: _Group("tp", [(p, t) for t in range(tp)]) for p in range(pp)}
        self.pp_groups = {t: _Group("pp", [(p, t) for p in range(pp)]) for t in range(tp)}
        self.dp_group = _Group("dp", [0])

    def context(self, p, t):
        rank = (p * self.dp) * self.tp + t
        return ParallelContext(
            rank=rank, world_size=self.tp * self.pp * self.dp, tp_size=self.tp, tp_rank=t,
            pp_size=self.pp, pp_rank=p, dp_size=self.dp, dp_rank=0,
            tp_group=self.tp_groups[p], pp_group=self.pp_groups[t], dp_group=self.dp_group,
            tp_ranks=tuple(p * self.dp * self.tp + i for i in range(self.tp)),
            pp_ranks=tuple(i * self.dp * self.tp + t for i in range(self.pp)),
            dp_ranks=tuple(p * self.dp * self.tp + d * self.tp + t for d in range(self.dp)))

    def all_reduce(self, tensor, op=None, group=None, **_):
        me = self.local.coord
        if group.kind == "dp":
            self.dp_calls.append(me)
            raise AssertionError("gradient-norm terms were reduced over data parallelism")
        self.log.append((me, group.kind))
        group.slots[me] = tensor.clone()
        group.barrier.wait()
        total = sum(group.slots[m] for m in group.members)
        group.barrier.wait()
        tensor.copy_(total)

    def run(self, fn):
        """``fn(p, t, ctx)`` on every virtual rank at once; results by coordinate."""
        results, errors = {}, []

        def body(p, t):
            self.local.coord = (p, t)
            try:
                results[p, t] = fn(p, t, self.context(p, t))
            except BaseException as exc:  # noqa: BLE001 - reported below
                errors.append(exc)
                for g in (self.tp_groups[p], self.pp_groups[t]):
                    g.barrier.abort()

        threads = [threading.Thread(target=body, args=(p, t))
                   for p in range(self.pp) for t in range(self.tp)]
        for th in threads:
            th.start()
        for th in threads:
            th.join(timeout=30)
        if errors:
            raise errors[0]
        return results


@contextmanager
def simulated(world):
    original = grads.dist.all_reduce
    grads.dist.all_reduce = world.all_reduce
    try:
        yield world
    finally:
        grads.dist.all_reduce = original


class _Param(nn.Module):
    def __init__(self, grad, sharded):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros_like(grad))
        self.weight.grad = grad.clone()
        self.weight.tensor_parallel_sharded = sharded


def _logical(pp, tp, seed=7):
    """Unsharded logical gradients of a stage stack with tied embedding / LM head."""
    g = torch.Generator().manual_seed(seed)
    return {
        "attn": [torch.randn(6, 4 * tp, generator=g) for _ in range(pp)],  # column-sharded per stage
        "norm": [torch.randn(6, generator=g) for _ in range(pp)],          # replicated per stage
        "embedding": torch.randn(8 * tp, 6, generator=g),                  # vocab-sharded, tied
    }


def _stage(logical, p, t, tp, pp, tied):
    m = nn.Module()
    m.attn = _Param(logical["attn"][p][:, 4 * t: 4 * t + 4], True)
    m.norm = _Param(logical["norm"][p], False)
    shard = logical["embedding"][8 * t: 8 * t + 8]
    if p == 0:
        m.embedding = _Param(shard, True)
    if p == pp - 1 and (pp > 1 or not tied):
        m.lm_head = _Param(shard if tied else shard * 0.5, True)
    return m


def _expected_norm(logical, pp, tied):
    sq = sum(a.double().pow(2).sum() for a in logical["attn"])
    sq += sum(n.double().pow(2).sum() for n in logical["norm"])
    sq += logical["embedding"].double().pow(2).sum()
    if not tied:
        sq += (logical["embedding"] * 0.5).double().pow(2).sum()
    return sq.sqrt()


@pytest.mark.parametrize("tp, pp, tied", [(2, 2, True), (4, 2, True), (2, 3, False), (1, 2, True)])
def test_logical_norm_and_uniform_scaling(tp, pp, tied):
    logical = _logical(pp, tp)
    expected = _expected_norm(logical, pp, tied)
    max_norm = float(expected) / 3

    def rank_fn(p, t, ctx):
        stage = _stage(logical, p, t, tp, pp, tied)
        before = {n: q.grad.clone() for n, q in stage.named_parameters()}
        norm = grads.clip_grad_norm(stage, ctx, max_norm, tie_embeddings=tied)
        ratios = {n: q.grad / before[n] for n, q in stage.named_parameters()}
        return norm, ratios

    with simulated(ThreadWorld(tp, pp)) as world:
        results = world.run(rank_fn)
    coefficient = max_norm / (float(expected) + 1e-6)
    for (norm, ratios) in results.values():
        torch.testing.assert_close(norm, expected, rtol=1e-12, atol=0)
        for r in ratios.values():
            torch.testing.assert_close(r, torch.full_like(r, coefficient), rtol=1e-6, atol=0)
    kinds = [k for _, k in world.log]
    assert kinds.count("tp") == (tp * pp if tp > 1 else 0)
    assert kinds.count("pp") == (tp * pp if pp > 1 else 0)
    assert world.dp_calls == []


def test_small_norm_leaves_gradients_alone_and_zero_limit_clears_them():
    logical = _logical(1, 1, seed=3)
    expected = _expected_norm(logical, 1, True)
    for limit, factor in ((float(expected) * 10, 1.0), (0.0, 0.0)):
        def rank_fn(p, t, ctx):
            stage = _stage(logical, p, t, 1, 1, True)
            before = [q.grad.clone() for q in stage.parameters()]
            norm = grads.clip_grad_norm(stage, ctx, limit, tie_embeddings=True)
            return norm, [(q.grad, b * factor) for q, b in zip(stage.parameters(), before)]
        with simulated(ThreadWorld(1, 1)) as world:
            (norm, pairs), = world.run(rank_fn).values()
        torch.testing.assert_close(norm, expected)
        for got, want in pairs:
            assert torch.equal(got, want)


def test_parameters_without_gradients_and_negative_limit():
    m = nn.Module()
    m.weight = nn.Parameter(torch.ones(3))
    assert grads.clip_grad_norm(m, ParallelContext.single(), 1.0).item() == 0.0
    with pytest.raises(ValueError, match="non-negative"):
        grads.clip_grad_norm(m, ParallelContext.single(), -0.5)


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
