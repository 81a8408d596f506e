"""Rank-local training checkpoints with a completion manifest and integrity data.

Directory of one saved step (the layout of ``nano_megatron/checkpoint.py``,
kept so tools and resume scripts find the same files)::

    rank_{global_rank:05d}.pt   one shard per rank
    manifest.pt                 rank 0 writes it last; a directory without it is incomplete

A shard is a dict with the keys ``version``, ``topology``, ``model``,
``model_config``, ``optimizer``, ``step``, ``rng``, ``data`` and ``extra``.
The manifest carries ``version``, ``step``, ``world_size``,
``parallel_sizes`` and ``shards`` and, in this implementation, the byte size
and CRC-32 of every shard, so a resumed run detects a truncated or damaged
shard instead of loading it.

Saving (a collective over the world when it has more than one rank):

1. rank 0 withdraws an existing manifest, and every rank waits for that, so a
   crash from here on leaves the directory visibly incomplete;
2. every rank streams its shard through a CRC-32 counter into a temporary
   file of the same directory, ``fsync``s it and renames it into place;
3. the (size, CRC) pairs are gathered to rank 0, which writes the manifest the
   same durable way; every rank waits for it before returning.

Loading checks, before it changes any state: the manifest can be read; its
version, world size and parallel sizes match this run; every listed shard
exists; this rank's shard has the recorded size and CRC; the shard's version,
topology, model configuration and step agree with the manifest and the run;
and a data stream is supplied if the shard holds a stream position. All
failing checks are reported together in one :class:`CheckpointError`.
"""

from __future__ import annotations

import io
import os
import random
import tempfile
import zlib
from dataclasses import asdict, is_dataclass
from pathlib import Path

import torch

from ..parallel.context import ParallelContext

FORMAT_VERSION = 1
MANIFEST = "manifest.pt"


class CheckpointError(RuntimeError):
    """A checkpoint directory that cannot be written or resumed by this run."""


def shard_name(rank: int) -> str:
    return f"rank_{rank:05d}.pt"


def topology(ctx: ParallelContext) -> dict[str, int]:
    """The rank coordinates a shard is valid for."""
    return {"world_size": ctx.world_size, "global_rank": ctx.rank,
            "tp_size": ctx.tp_size, "tp_rank": ctx.tp_rank,
            "pp_size": ctx.pp_size, "pp_rank": ctx.pp_rank,
            "dp_size": ctx.dp_size, "dp_rank": ctx.dp_rank}


def _sizes(ctx: ParallelContext) -> dict[str, int]:
    return {"tp": ctx.tp_size, "pp": ctx.pp_size, "dp": ctx.dp_size}


class _Checksummed(io.RawIOBase):
    """Write-through file wrapper that counts bytes and folds them into a CRC-32."""

    def __init__(self, raw):
        self.raw, self.crc, self.size = raw, 0, 0

    def writable(self) -> bool:
        return True

    def write(self, data) -> int:
        view = memoryview(data)
        self.raw.write(view)
        self.crc = zlib.crc32(view, self.crc)
        self.size += view.nbytes
        return view.nbytes


def _durable_save(obj, path: Path) -> dict[str, int]:
    """``torch.save`` into a temp file beside ``path``, fsync, rename; (size, crc) of the bytes."""
    fd, tmp = tempfile.mkstemp(prefix=f".{path.name}.", suffix=".partial", dir=path.parent)
    try:
        with os.fdopen(fd, "wb") as raw:
            sink = _Checksummed(raw)
            try:
                torch.save(obj, sink)
            except RuntimeError as exc:
                # torch's zip writer replaces a failed write with its own error
                # when it closes; report the I/O error the caller can act on
                if isinstance(exc.__context__, OSError):
                    raise exc.__context__ from exc
                raise
            raw.flush()
            os.fsync(raw.fileno())
        os.replace(tmp, path)
    except BaseException:
        Path(tmp).unlink(missing_ok=True)
        raise
    dir_fd = os.open(path.parent, os.O_RDONLY)
    try:  # make the rename itself durable
        os.fsync(dir_fd)
    finally:
        os.close(dir_fd)
    return {"bytes": sink.size, "crc32": sink.crc}


def _host_copy(obj):
    """Deep copy with every tensor on the host, so a shard never pins device memory."""
    if torch.is_tensor(obj):
        return obj.detach().to("cpu", copy=True)
    if isinstance(obj, dict):
        return {k: _host_copy(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_host_copy(v) for v in obj)
    return obj


def _random_states() -> dict:
    states = {"cpu": torch.get_rng_state(), "python": random.getstate()}
    if torch.cuda.is_available():
        states["cuda"] = torch.cuda.get_rng_state_all()
    return states


def _apply_random_states(states: dict) -> None:
    torch.set_rng_state(states["cpu"])
    random.setstate(states["python"])
    if "cuda" in states:
        torch.cuda.set_rng_state_all(states["cuda"])


def _model_config(model):
    config = getattr(model, "config", None)
    return asdict(config) if config is not None and is_dataclass(config) else None


def _valid_step(step) -> bool:
    return type(step) is int and step >= 0


def save_checkpoint(directory, model, optimizer, ctx: ParallelContext, *, step: int,
                    data=None, extra: dict | None = None) -> Path:
    """Write this rank's shard (and, on rank 0, the manifest) into ``directory``.

    Collective when the world has more than one rank. Returns the shard path.
    """
    if not _valid_step(step):
        raise ValueError(f"save_checkpoint: step {step!r} is not a non-negative int")
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    group_save = ctx.world_size > 1 and torch.distributed.is_initialized()
    manifest_path = directory / MANIFEST

    if ctx.rank == 0:
        manifest_path.unlink(missing_ok=True)
    if group_save:
        torch.distributed.barrier()

    shard = {
        "version": FORMAT_VERSION, "topology": topology(ctx),
        "model": _host_copy(model.state_dict()), "model_config": _model_config(model),
        "optimizer": _host_copy(optimizer.state_dict()), "step": step,
        "rng": _random_states(), "data": None if data is None else data.state_dict(),
        "extra": dict(extra or {}),
    }
    path = directory / shard_name(ctx.rank)
    digest = _durable_save(shard, path)

    digests = [None] * ctx.world_size
    if group_save:
        torch.distributed.all_gather_object(digests, digest)
    else:
        digests[0] = digest
    if ctx.rank == 0:
        names = [shard_name(r) for r in range(ctx.world_size)]
        absent = [n for n in names if not (directory / n).is_file()]
        if absent:
            raise CheckpointError(f"{directory}: shards {absent} were not written; no manifest")
        _durable_save({"version": FORMAT_VERSION, "step": step, "world_size": ctx.world_size,
                       "parallel_sizes": _sizes(ctx), "shards": names,
                       "shard_digests": dict(zip(names, digests))}, manifest_path)
    if group_save:
        torch.distributed.barrier()
    return path


def _read(path: Path, what: str, map_location, problems: list[str], digest=None):
    try:
        blob = path.read_bytes()
    except OSError as exc:
        problems.append(f"{what} {path.name} cannot be read ({exc.strerror})")
        return None
    if digest is not None:
        if len(blob) != digest["bytes"]:
            problems.append(f"{what} {path.name} has {len(blob)} bytes, the manifest recorded "
                            f"{digest['bytes']} (truncated or overwritten)")
            return None
        if zlib.crc32(blob) != digest["crc32"]:
            problems.append(f"{what} {path.name} fails its CRC-32 check (damaged)")
            return None
    try:
        obj = torch.load(io.BytesIO(blob), map_location=map_location, weights_only=False)
    except Exception as exc:  # torch raises several types for a damaged zip/pickle
        problems.append(f"{what} {path.name} is not a readable torch file ({type(exc).__name__})")
        return None
    if not isinstance(obj, dict):
        problems.append(f"{what} {path.name} does not hold a dict")
        return None
    return obj


def _fail(directory: Path, problems: list[str]):
    raise CheckpointError(f"cannot resume from {directory}:\n  - " + "\n  - ".join(problems))


def load_checkpoint(directory, model, optimizer, ctx: ParallelContext, *, data=None,
                    map_location="cpu") -> tuple[int, dict]:
    """Validate ``directory`` for this rank, then restore model, optimizer, RNG and
    data position. Returns ``(step, extra)``. Nothing is modified unless every
    check passes."""
    directory = Path(directory)
    problems: list[str] = []
    manifest_path = directory / MANIFEST
    if not manifest_path.is_file():
        _fail(directory, ["no manifest.pt: the save did not complete"])
    manifest = _read(manifest_path, "manifest", "cpu", problems)
    if manifest is None:
        _fail(directory, problems)

    table = [("format version", manifest.get("version"), FORMAT_VERSION),
             ("world size", manifest.get("world_size"), ctx.world_size),
             ("parallel sizes", manifest.get("parallel_sizes"), _sizes(ctx))]
    problems += [f"{name}: checkpoint {saved!r}, this run {now!r}" for name, saved, now in table
                 if saved != now]
    listed = list(manifest.get("shards") or ())
    missing = [n for n in listed if not (directory / n).is_file()]
    if missing:
        problems.append(f"listed shards missing on disk: {missing}")
    if not _valid_step(manifest.get("step")):
        problems.append(f"manifest step {manifest.get('step')!r} is not a non-negative int")
    if problems:
        _fail(directory, problems)

    mine = shard_name(ctx.rank)
    digest = (manifest.get("shard_digests") or {}).get(mine)
    shard = _read(directory / mine, "shard", map_location, problems, digest)
    if shard is None:
        _fail(directory, problems)
    table = [("shard format version", shard.get("version"), FORMAT_VERSION),
             ("rank topology", shard.get("topology"), topology(ctx)),
             ("model configuration", shard.get("model_config"), _model_config(model)),
             ("step (shard vs manifest)", shard.get("step"), manifest["step"])]
    problems += [f"{name}: checkpoint {saved!r}, expected {now!r}" for name, saved, now in table
                 if saved != now]
    if shard.get("data") is not None and data is None:
        problems.append("the shard holds a data-stream position but no stream was passed")
    if "cuda" in (shard.get("rng") or {}) and not torch.cuda.is_available():
        problems.append("the shard holds CUDA generator states but CUDA is not available")
    if problems:
        _fail(directory, problems)

    model.load_state_dict(shard["model"])
    optimizer.load_state_dict(shard["optimizer"])
    if shard["data"] is not None:
        data.load_state_dict(shard["data"])
    _apply_random_states(shard["rng"])
    return shard["step"], shard.get("extra") or {}
