"""Reshard a checkpoint to another tensor / pipeline / data-parallel layout,
offline, on the CPU:

    python -m nano_megatron_b200.utils.reshard SRC_STEP_DIR DST_STEP_DIR --tp T --pp P [--dp D]

A step directory written by :func:`~nano_megatron_b200.utils.checkpoint.save_checkpoint`
holds, per rank, that rank's slice of every parameter and of its two AdamW
moments (flat buffers in the stage's layout). This tool rebuilds every
logical parameter and moment from the source shards, cuts them for each rank
of the target layout and writes a complete step directory (shards, then the
manifest with their sizes and CRC-32s) that ``load_checkpoint`` resumes at
the new layout.

How a tensor is cut follows from the layer that owns it: column-parallel
weights along dim 1 (their bias along dim 0), row-parallel weights and the
vocabulary-sharded embedding and LM head along dim 0; everything else (the
norms, row-parallel biases) is replicated and must agree across TP ranks
(to fp32 rounding; TP rank 0's copy is written).
Layer ``i`` of pipeline stage ``p`` is global layer ``p * L / pp + i``. DP
replicas hold identical model and optimizer state (gradients are averaged
before every step), so the first replica of each (tp, pp) position is read.

Kept: the step, the optimizer's step count and hyperparameters, ``extra``
(the training settings) and the token stream's global cursor, whose layout
entry takes the target rank's DP coordinates. Generator states come from the
source rank with the same global rank (rank 0 for ranks the source lacked):
a random stream has no continuation across layouts.

The reference's checkpoints are valid only for the layout that wrote them
(``nano_megatron/checkpoint.py:129-196``); changing the layout is an addition.
Memory: every logical parameter with its two moments is held at once (three
fp32 copies of the model), plus one stage model at a time.
"""

from __future__ import annotations

import argparse
from pathlib import Path

import torch

from ..models import GPT, GPTConfig
from ..models.gpt import ParallelLMHead
from ..models.layers import ColumnParallelLinear, RowParallelLinear, VocabParallelEmbedding
from ..optim import FusedAdamW
from ..parallel.context import ParallelContext, grid_ranks
from . import checkpoint as ckpt


def contexts(tp: int, pp: int, dp: int) -> list[ParallelContext]:
    """Every rank's coordinates of a layout (no process groups: offline use)."""
    world = tp * pp * dp
    grid, _ = grid_ranks(world, tp, pp)
    out = []
    for p in range(pp):
        for d in range(dp):
            for t in range(tp):
                out.append(ParallelContext(
                    rank=grid[p][d][t], world_size=world, tp_size=tp, tp_rank=t, pp_size=pp, pp_rank=p,
                    dp_size=dp, dp_rank=d, tp_ranks=tuple(grid[p][d]),
                    pp_ranks=tuple(grid[q][d][t] for q in range(pp)),
                    dp_ranks=tuple(grid[p][e][t] for e in range(dp))))
    return sorted(out, key=lambda c: c.rank)


def split_dims(model) -> dict[str, int | None]:
    """Parameter name -> the dim TP ranks split it along (None: replicated)."""
    dims: dict[str, int | None] = {}
    for mname, module in model.named_modules():
        prefix = f"{mname}." if mname else ""
        if isinstance(module, ColumnParallelLinear):
            dims[prefix + "weight"] = 1
            if module.bias is not None:
                dims[prefix + "bias"] = 0
        elif isinstance(module, RowParallelLinear):
            dims[prefix + "weight"] = 0
        elif isinstance(module, (VocabParallelEmbedding, ParallelLMHead)):
            dims[prefix + "weight"] = 0
    return {name: dims.get(name) for name, _ in model.named_parameters()}


def _global_name(name: str, pp_rank: int, layers_per_stage: int) -> str:
    parts = name.split(".")
    if parts[0] == "layers":
        parts[1] = str(pp_rank * layers_per_stage + int(parts[1]))
    return ".".join(parts)


def _moment_views(model, optimizer: FusedAdamW):
    """``name -> (exp_avg view, exp_avg_sq view)`` shaped like each parameter."""
    base = optimizer.flat.data.storage_offset()
    views = {}
    for name, p in model.named_parameters():
        offset = p.data.storage_offset() - base
        views[name] = tuple(torch.as_strided(flat, p.shape, p.stride(), offset)
                            for flat in (optimizer.exp_avg, optimizer.exp_avg_sq))
    return views


def _stage(config: GPTConfig, ctx: ParallelContext):
    model = GPT(config, ctx)
    return model, FusedAdamW(model)


def _read_step(src: Path):
    problems: list[str] = []
    manifest = ckpt._read(src / ckpt.MANIFEST, "manifest", "cpu", problems)
    if manifest is None:
        ckpt._fail(src, [ckpt._no_manifest(src)] if not (src / ckpt.MANIFEST).exists() else problems)
    if manifest.get("version") != ckpt.FORMAT_VERSION:
        ckpt._fail(src, [f"format version {manifest.get('version')!r}: this tool reads "
                         f"{ckpt.FORMAT_VERSION} (save_checkpoint's format)"])
    sizes = manifest.get("parallel_sizes") or {}
    shards = {}
    for rank in range(manifest.get("world_size", 0)):
        name = ckpt.shard_name(rank)
        digest = (manifest.get("shard_digests") or {}).get(name)
        shard = ckpt._read(src / name, "shard", "cpu", problems, digest)
        if shard is not None:
            if shard.get("step") != manifest.get("step"):
                problems.append(f"{name}: step {shard.get('step')!r}, manifest {manifest.get('step')!r}")
            shards[rank] = shard
    configs = {repr(s.get("model_config")) for s in shards.values()}
    if len(configs) > 1:
        problems.append("the shards hold different model configurations")
    layout = (sizes.get("tp"), sizes.get("pp"), sizes.get("dp"))
    if not all(isinstance(n, int) and n > 0 for n in layout) or layout[0] * layout[1] * layout[2] != len(shards):
        problems.append(f"parallel sizes {sizes!r} do not describe {len(shards)} shards")
    else:
        for ctx in contexts(*layout):
            saved = shards[ctx.rank].get("topology") if ctx.rank in shards else None
            if saved != ckpt.topology(ctx):
                problems.append(f"{ckpt.shard_name(ctx.rank)}: topology {saved!r}, the manifest's layout "
                                f"gives {ckpt.topology(ctx)!r}")
    if problems:
        ckpt._fail(src, problems)
    return manifest, layout, shards


def _logical_state(config: GPTConfig, layout, shards):
    """``global name -> [value, exp_avg, exp_avg_sq]`` (full tensors) and the
    optimizer state shared by all ranks."""
    tp, pp, dp = layout
    layers_per_stage = config.n_layer // pp
    pieces: dict[str, list] = {}
    dims: dict[str, int | None] = {}
    opt_meta = None
    for ctx in contexts(tp, pp, dp):
        if ctx.dp_rank != 0:
            continue
        shard = shards[ctx.rank]
        model, opt = _stage(config, ctx)
        model.load_state_dict(shard["model"])
        opt.load_state_dict(shard["optimizer"])
        meta = (opt.step_count, opt.param_groups)
        if opt_meta is None:
            opt_meta = meta
        elif meta != opt_meta:
            raise ckpt.CheckpointError(f"rank {ctx.rank}: optimizer step or hyperparameters differ from rank 0")
        moments = _moment_views(model, opt)
        params = dict(model.named_parameters())
        for name, dim in split_dims(model).items():
            key = _global_name(name, ctx.pp_rank, layers_per_stage)
            triple = [params[name].detach().clone(), *(m.clone() for m in moments[name])]
            dims[key] = dim
            slots = pieces.setdefault(key, [None] * tp)
            slots[ctx.tp_rank] = triple
    logical = {}
    for key, slots in pieces.items():
        dim = dims[key]
        if dim is None:
            first = slots[0]
            for t, other in enumerate(slots[1:], 1):
                if any(not torch.allclose(a, b, rtol=1e-5, atol=1e-7) for a, b in zip(first, other)):
                    raise ckpt.CheckpointError(f"replicated parameter {key} differs between TP ranks 0 and {t}")
            logical[key] = first
        else:
            logical[key] = [torch.cat([s[i] for s in slots], dim=dim) for i in range(3)]
    return logical, opt_meta


def reshard(src, dst, tp: int, pp: int, dp: int = 1) -> Path:
    """Write ``src`` (a step directory) into ``dst`` for a TP x PP x DP layout;
    returns ``dst``. Nothing is written when the source fails its checks or
    the model does not divide over the target layout."""
    src, dst = Path(src), Path(dst)
    if dst.resolve() == src.resolve():
        raise ValueError(f"reshard writes a new step directory; {dst} is the source")
    manifest, layout, shards = _read_step(src)
    config = GPTConfig(**shards[0]["model_config"])
    targets = contexts(tp, pp, dp)
    for ctx in targets[:1]:
        GPT(config, ctx)  # raises if the model does not divide over the target layout
    logical, (step_count, param_groups) = _logical_state(config, layout, shards)
    tied = config.tie_word_embeddings
    layers_per_stage = config.n_layer // pp

    out = []
    for ctx in targets:
        model, opt = _stage(config, ctx)
        opt.step_count = step_count
        opt.param_groups = [dict(g) for g in param_groups]
        moments = _moment_views(model, opt)
        params = dict(model.named_parameters())
        with torch.no_grad():
            for name, dim in split_dims(model).items():
                key = _global_name(name, ctx.pp_rank, layers_per_stage)
                if key not in logical and tied and key == "lm_head.weight":
                    key = "embedding.weight"  # one tied tensor in the source, two copies here
                full = logical[key]
                part = [f if dim is None else f.chunk(tp, dim=dim)[ctx.tp_rank] for f in full]
                params[name].copy_(part[0])
                moments[name][0].copy_(part[1])
                moments[name][1].copy_(part[2])
        model.refresh_compute_copies()
        template = shards.get(ctx.rank, shards[0])
        data = shards[0].get("data")
        if data is not None:
            data = dict(data, layout=dict(data["layout"], dp_rank=ctx.dp_rank, dp_size=dp))
        out.append({
            "version": ckpt.FORMAT_VERSION, "topology": ckpt.topology(ctx),
            "model": ckpt._host_copy(model.state_dict()), "model_config": shards[0]["model_config"],
            "optimizer": ckpt._host_copy(opt.state_dict()), "step": manifest["step"],
            "rng": template["rng"], "data": data, "extra": dict(shards[0].get("extra") or {}),
        })

    dst.mkdir(parents=True, exist_ok=True)
    (dst / ckpt.MANIFEST).unlink(missing_ok=True)
    names = [ckpt.shard_name(r) for r in range(len(out))]
    digests = {name: ckpt._durable_save(shard, dst / name) for name, shard in zip(names, out)}
    ckpt._durable_save({"version": ckpt.FORMAT_VERSION, "step": manifest["step"], "world_size": len(out),
                        "parallel_sizes": {"tp": tp, "pp": pp, "dp": dp}, "shards": names,
                        "shard_digests": digests}, dst / ckpt.MANIFEST)
    return dst


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Reshard a checkpoint step directory to another TP x PP x DP layout.")
    p.add_argument("src", help="step directory written by save_checkpoint")
    p.add_argument("dst", help="step directory to write")
    p.add_argument("--tp", type=int, required=True)
    p.add_argument("--pp", type=int, required=True)
    p.add_argument("--dp", type=int, default=1)
    args = p.parse_args(argv)
    out = reshard(args.src, args.dst, args.tp, args.pp, args.dp)
    print(f"wrote {out} for tp={args.tp} pp={args.pp} dp={args.dp}")


if __name__ == "__main__":
    main()
