"""Socket-free checks: sharding rules cover every parameter, shard/concat
round-trips, stage partition is exact, the pp=1 tie shares storage, gradient
sync tags match the rules, fused QKV / gate|up weights are views of one region."""

import torch

from nano_megatron_b200.models import GPTConfig, layers_for_stage
from tests.oracle import SHARD_DIM, full_model, shard_dim

CONFIG = GPTConfig(vocab_size=128, n_layer=4, n_head=4, n_embd=64, seq_len=16)


def test_full_model_runs_with_all_grads():
    model = full_model(CONFIG)
    x = torch.randint(0, CONFIG.vocab_size, (2, CONFIG.seq_len))
    y = torch.randint(0, CONFIG.vocab_size, (2, CONFIG.seq_len))
    loss = model(x, y)
    loss.backward()
    assert torch.isfinite(loss)
    assert all(p.grad is not None and p.grad.abs().sum() > 0 for p in model.parameters())


def test_every_parameter_has_a_rule():
    model = full_model(CONFIG)
    unclassified = [n for n, _ in model.named_parameters()
                    if shard_dim(n) is None and not n.endswith(("norm.weight", ".bias"))]
    assert not unclassified, unclassified
    assert len(SHARD_DIM) == 9


def test_shard_concat_roundtrip():
    model = full_model(CONFIG)
    checked = 0
    for name, p in model.named_parameters():
        dim = shard_dim(name)
        if dim is None:
            continue
        for tp in (2, 4):
            if p.shape[dim] % tp == 0:
                assert torch.equal(torch.cat(torch.chunk(p.data, tp, dim=dim), dim=dim), p.data)
                checked += 1
    assert checked > 0


def test_layer_partition_exact():
    for pp in (1, 2, 4):
        covered = [i for r in range(pp) for i in range(*layers_for_stage(CONFIG.n_layer, pp, r))]
        assert covered == list(range(CONFIG.n_layer))


def test_tied_embedding_shares_storage():
    model = full_model(CONFIG)
    assert model.lm_head.weight is model.embedding.weight


def test_sync_tags_match_rules():
    model = full_model(CONFIG)
    for name, p in model.named_parameters():
        assert getattr(p, "tensor_parallel_sharded", False) == (shard_dim(name) is not None), name


def test_fused_projections_are_views_of_flat_buffer():
    model = full_model(CONFIG)
    attn = model.layers[0].attn
    region = model.flat_buffers.region_of(attn.q.weight)
    assert region.shape == (64, 192)
    assert attn.q.weight.data_ptr() == region.data_block.data_ptr()
    assert attn.k.weight.data_ptr() == region.data_block.data_ptr() + 64 * 4
    mlp = model.layers[0].mlp
    assert model.flat_buffers.region_of(mlp.up.weight).shape == (64, 2 * 256)
    for p in model.parameters():
        assert p.grad is p.main_grad or p.grad.data_ptr() == p.main_grad.data_ptr()
        base = model.flat_buffers.data.data_ptr()
        assert base <= p.data_ptr() < base + model.flat_buffers.data.numel() * 4
