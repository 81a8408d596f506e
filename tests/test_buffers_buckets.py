"""Flat buffers and the data-parallel bucketer, single process on CPU.

* ``FlatBuffers.rehome_grad`` moves the gradient into a new buffer and every
  view (parameter ``.grad`` / ``main_grad``, region blocks) follows it.
* ``GradBucketer`` cuts the buffer into buckets of whole regions that cover
  every element exactly once, formed from the end of the buffer; it learns the
  writes per region from the earlier microbatches (two for an embedding tied to
  the LM head) and starts a bucket once all its regions are complete.
"""

import pytest
import torch
import torch.distributed as dist

from nano_megatron_b200.models import GPT, GPTConfig
from nano_megatron_b200.models.functional import set_grad_observer
from nano_megatron_b200.parallel import init_parallel
from nano_megatron_b200.parallel.grads import GradBucketer
from nano_megatron_b200.parallel.pipeline import forward_backward_1f1b


def _model(tie=True):
    cfg = GPTConfig(vocab_size=64, n_layer=3, n_head=2, n_embd=32, seq_len=8, tie_word_embeddings=tie)
    torch.manual_seed(0)
    return cfg, GPT(cfg)


def test_rehome_grad_moves_every_view():
    _, model = _model()
    flat = model.flat_buffers
    flat.grad.normal_()
    before = flat.grad.clone()
    new = torch.empty_like(flat.grad)
    flat.rehome_grad(new)
    assert flat.grad.data_ptr() == new.data_ptr()
    assert torch.equal(flat.grad, before)
    for region in flat.regions:
        assert region.grad_block.untyped_storage().data_ptr() == new.untyped_storage().data_ptr()
        for p in region.params:
            assert p.grad.untyped_storage().data_ptr() == new.untyped_storage().data_ptr()
            assert p.main_grad is p.grad
    model.layers[0].mlp.down.weight.grad.fill_(3.0)
    region = flat.region_of(model.layers[0].mlp.down.weight)
    assert torch.all(new[region.offset: region.offset + region.numel] == 3.0)


@pytest.fixture
def single_rank_group(tmp_path):
    """A one-rank Gloo process group for the duration of one test."""
    dist.init_process_group("gloo", init_method=f"file://{tmp_path}/rdzv", rank=0, world_size=1)
    yield init_parallel(1, 1)
    dist.destroy_process_group()


@pytest.mark.distributed
def test_buckets_cover_the_buffer_once_from_the_end(single_rank_group):
    ctx = single_rank_group
    _, model = _model()
    flat = model.flat_buffers
    for size in (1, 4096, 64 << 10, 1 << 30):
        b = GradBucketer(model, ctx, bucket_bytes=size)
        spans = sorted(b.buckets)
        assert spans[0][0] == 0 and spans[-1][1] == flat.numel
        assert all(a[1] == c[0] for a, c in zip(spans, spans[1:]))  # contiguous, no overlap
        assert b.bucket_regions[0][0] == len(flat.regions) - 1       # first bucket holds the last region
        assert sorted(r for rs in b.bucket_regions for r in rs) == list(range(len(flat.regions)))


@pytest.mark.distributed
def test_bucketer_learns_writes_and_starts_buckets_during_last_backward(single_rank_group):
    ctx = single_rank_group
    cfg, model = _model(tie=True)
    bucketer = GradBucketer(model, ctx, bucket_bytes=2048)
    started_at_last = []
    set_grad_observer(bucketer.observe)
    try:
        gen = torch.Generator().manual_seed(1)
        batches = [(torch.randint(0, 64, (1, 8), generator=gen), torch.randint(0, 64, (1, 8), generator=gen))
                   for _ in range(3)]

        def hook(prior):
            bucketer.before_last_backward(prior)
            started_at_last.append(sum(bucketer.started))

        forward_backward_1f1b(model, batches, cfg, "cpu", ctx, before_last_backward=hook)
        started_in_backward = sum(bucketer.started)
        emb = model.flat_buffers.regions.index(model.flat_buffers.region_of(model.embedding.weight))
        assert bucketer.per_microbatch[emb] == 2  # the tied embedding: LM head and embedding backward
        assert all(w >= 1 for w in bucketer.per_microbatch)
        assert started_in_backward == len(bucketer.buckets)  # every bucket completed during the last backward
        assert started_at_last == [0]
        bucketer.finish()
    finally:
        set_grad_observer(None)
