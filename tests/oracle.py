"""Unsharded-model oracle: build one full model and slice it per rank.

The sharding rules (which reference dim each parameter is split along across
the TP group; anything unlisted is replicated) are written down here once. If
the distributed tests pass, these rules and the layers agree.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from nano_megatron_b200.models import GPT, GPTConfig, layers_for_stage
from nano_megatron_b200.parallel import ParallelContext

SHARD_DIM = {
    "attn.q.weight": 1, "attn.k.weight": 1, "attn.v.weight": 1, "attn.proj.weight": 0,
    "mlp.gate.weight": 1, "mlp.up.weight": 1, "mlp.down.weight": 0,
    "embedding.weight": 0, "lm_head.weight": 0,
}


def shard_dim(name: str):
    for suffix, dim in SHARD_DIM.items():
        if name.endswith(suffix):
            return dim
    return None


def full_model(config: GPTConfig, seed: int = 0) -> GPT:
    torch.manual_seed(seed)
    return GPT(config, ParallelContext.single())


def shard_state(full: GPT, config: GPTConfig, ctx: ParallelContext) -> dict:
    start, end = layers_for_stage(config.n_layer, ctx.pp_size, ctx.pp_rank)
    out = {}
    for name, tensor in full.state_dict().items():
        if name.startswith("layers."):
            _, idx, rest = name.split(".", 2)
            if not start <= int(idx) < end:
                continue
            local = f"layers.{int(idx) - start}.{rest}"
        elif name.startswith("embedding."):
            if not ctx.is_first_stage:
                continue
            local = name
        elif name.startswith(("lm_head.", "final_norm.")):
            if not ctx.is_last_stage:
                continue
            local = name
        else:
            continue
        dim = shard_dim(name)
        if dim is None or ctx.tp_size == 1:
            out[local] = tensor.clone()
        else:
            out[local] = torch.chunk(tensor, ctx.tp_size, dim=dim)[ctx.tp_rank].contiguous()
    return out


def parallel_model(config: GPTConfig, full: GPT, ctx: ParallelContext) -> GPT:
    model = GPT(config, ctx)
    missing, unexpected = model.load_state_dict(shard_state(full, config, ctx), strict=False)
    if unexpected or missing:
        raise RuntimeError(f"sharding mismatch: missing={missing} unexpected={unexpected}")
    return model


def gather_tensor(name: str, tensor: torch.Tensor, ctx: ParallelContext) -> torch.Tensor:
    dim = shard_dim(name)
    if dim is None or ctx.tp_size == 1:
        return tensor.detach().clone()
    parts = [torch.empty(tensor.shape, dtype=tensor.dtype) for _ in range(ctx.tp_size)]
    dist.all_gather(parts, tensor.detach().contiguous(), group=ctx.tp_group)
    return torch.cat(parts, dim=dim)
