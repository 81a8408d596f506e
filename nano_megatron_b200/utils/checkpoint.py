"""Atomic, rank-local training checkpoints for a fixed parallel topology.

Layout of one checkpoint directory (``<save>/step_{n:08d}``)::

    rank_{rank:05d}.pt   one shard per global rank
    manifest.pt          written last by rank 0; its presence marks completion

Commit protocol: rank 0 removes a stale manifest -> barrier -> every rank
writes its shard to a temporary name and renames it into place -> barrier ->
rank 0 checks that all shards exist and writes the manifest the same way ->
barrier. Loading validates the manifest, every shard's presence, this shard's
version, topology, model config and step before it touches any state.

A shard holds: format version, topology, model state dict, model config,
optimizer state dict, step, RNG states (torch CPU, python, every CUDA device),
token-stream state and caller extras.

Parity: ``nano_megatron/checkpoint.py:16-196`` (same file names, keys,
protocol and validation order).
"""

from __future__ import annotations

import os
import random
from dataclasses import asdict, is_dataclass
from pathlib import Path

import torch

from ..parallel.context import ParallelContext

FORMAT_VERSION = 1
MANIFEST = "manifest.pt"


def topology(ctx: ParallelContext) -> dict[str, int]:
    return {"world_size": ctx.world_size, "global_rank": ctx.rank,
            "tp_size": ctx.tp_size, "tp_rank": ctx.tp_rank,
            "pp_size": ctx.pp_size, "pp_rank": ctx.pp_rank,
            "dp_size": ctx.dp_size, "dp_rank": ctx.dp_rank}


def _capture_rng() -> dict:
    state = {"torch": torch.get_rng_state(), "python": random.getstate()}
    if torch.cuda.is_available():
        state["cuda"] = torch.cuda.get_rng_state_all()
    return state


def _restore_rng(state: dict) -> None:
    torch.set_rng_state(state["torch"])
    random.setstate(state["python"])
    if "cuda" in state:
        if not torch.cuda.is_available():
            raise RuntimeError("checkpoint contains CUDA RNG state but CUDA is unavailable")
        torch.cuda.set_rng_state_all(state["cuda"])


def shard_path(directory, ctx: ParallelContext) -> Path:
    return Path(directory) / f"rank_{ctx.rank:05d}.pt"


def _config_dict(model):
    config = getattr(model, "config", None)
    return asdict(config) if config is not None and is_dataclass(config) else None


def _write_atomically(obj, path: Path) -> None:
    tmp = path.with_name(f".{path.name}.{os.getpid()}.tmp")
    try:
        torch.save(obj, tmp)
        os.replace(tmp, path)
    finally:
        tmp.unlink(missing_ok=True)


def _distributed(ctx: ParallelContext) -> bool:
    return ctx.world_size > 1 and torch.distributed.is_initialized()


def _cpu_state(obj):
    """Deep-copy tensors to CPU so a shard does not pin device memory on load."""
    if torch.is_tensor(obj):
        return obj.detach().to("cpu", copy=True)
    if isinstance(obj, dict):
        return {k: _cpu_state(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_cpu_state(v) for v in obj)
    return obj


def save_checkpoint(directory, model, optimizer, ctx: ParallelContext, *, step: int,
                    data=None, extra: dict | None = None) -> Path:
    """Atomically write this rank's shard (and, on rank 0, the manifest)."""
    if isinstance(step, bool) or not isinstance(step, int) or step < 0:
        raise ValueError(f"step must be a non-negative integer, got {step!r}")
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    path = shard_path(directory, ctx)
    state = {
        "version": FORMAT_VERSION,
        "topology": topology(ctx),
        "model": _cpu_state(model.state_dict()),
        "model_config": _config_dict(model),
        "optimizer": _cpu_state(optimizer.state_dict()),
        "step": step,
        "rng": _capture_rng(),
        "data": data.state_dict() if data is not None else None,
        "extra": extra or {},
    }
    distributed = _distributed(ctx)
    manifest_path = directory / MANIFEST
    if distributed:
        if ctx.rank == 0:
            manifest_path.unlink(missing_ok=True)
        torch.distributed.barrier()
    _write_atomically(state, path)
    if distributed:
        torch.distributed.barrier()
    if ctx.rank == 0:
        shards = [f"rank_{r:05d}.pt" for r in range(ctx.world_size)]
        if not all((directory / s).is_file() for s in shards):
            raise RuntimeError("checkpoint is missing one or more rank shards")
        _write_atomically({"version": FORMAT_VERSION, "step": step, "world_size": ctx.world_size,
                           "parallel_sizes": {"tp": ctx.tp_size, "pp": ctx.pp_size,
                                              "dp": ctx.dp_size},
                           "shards": shards}, manifest_path)
    if distributed:
        torch.distributed.barrier()
    return path


def load_checkpoint(directory, model, optimizer, ctx: ParallelContext, *, data=None,
                    map_location="cpu") -> tuple[int, dict]:
    """Validate everything, then restore this rank; return ``(step, extra)``."""
    directory = Path(directory)
    manifest_path = directory / MANIFEST
    if not manifest_path.is_file():
        raise RuntimeError(f"checkpoint is incomplete: missing {manifest_path}")
    manifest = torch.load(manifest_path, map_location="cpu", weights_only=False)
    expected = {"version": FORMAT_VERSION, "world_size": ctx.world_size,
                "parallel_sizes": {"tp": ctx.tp_size, "pp": ctx.pp_size, "dp": ctx.dp_size}}
    for key, want in expected.items():
        if manifest.get(key) != want:
            raise RuntimeError(f"checkpoint manifest mismatch for {key}: "
                               f"saved={manifest.get(key)!r}, current={want!r}")
    if not all((directory / s).is_file() for s in manifest.get("shards", ())):
        raise RuntimeError("checkpoint is incomplete: a rank shard is missing")
    state = torch.load(shard_path(directory, ctx), map_location=map_location, weights_only=False)
    if state.get("version") != FORMAT_VERSION:
        raise RuntimeError(f"unsupported checkpoint version {state.get('version')!r}; "
                           f"expected {FORMAT_VERSION}")
    if state.get("topology") != topology(ctx):
        raise RuntimeError(f"checkpoint topology mismatch: saved={state.get('topology')}, "
                           f"current={topology(ctx)}")
    if state.get("model_config") != _config_dict(model):
        raise RuntimeError(f"checkpoint model configuration mismatch: "
                           f"saved={state.get('model_config')}, current={_config_dict(model)}")
    step = state.get("step")
    if isinstance(step, bool) or not isinstance(step, int) or step < 0:
        raise RuntimeError(f"invalid checkpoint step {step!r}")
    if manifest.get("step") != step:
        raise RuntimeError("checkpoint manifest and rank shard have different steps")
    if state["data"] is not None and data is None:
        raise RuntimeError("checkpoint contains data state but no data stream was provided")

    model.load_state_dict(state["model"])
    optimizer.load_state_dict(state["optimizer"])
    if state["data"] is not None:
        data.load_state_dict(state["data"])
    _restore_rng(state["rng"])
    return step, state.get("extra", {})
