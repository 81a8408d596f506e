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
    return _write_step(Path(directory), ctx, step, FORMAT_VERSION, lambda: {
        "version": FORMAT_VERSION, "topology": topology(ctx),
        "model": _host_copy(model.state_dict()), "model_config": _model_config(model),
        "optimizer": _host_copy(optimizer.state_dict()), "step": step,
        "rng": _random_states(), "data": None if data is None else data.state_dict(),
        "extra": dict(extra or {}),
    })


def _write_step(directory: Path, ctx: ParallelContext, step: int, version: int, make_shard) -> Path:
    """The save protocol shared by both formats: withdraw the manifest, write
    every rank's shard durably, then the manifest with the shards' sizes and
    CRC-32s (readers that do not know those keys ignore them)."""
    directory.mkdir(parents=True, exist_ok=True)
    group_save = ctx.world_size > 1 and torch.distributed.is_initialized()
    manifest_path = directory / MANIFEST

    if ctx.rank == 0:
        manifest_path.unlink(missing_ok=True)
    if group_save:
        torch.distributed.barrier()

    shard = make_shard()
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
        _durable_save({"version": version, "step": step, "world_size": ctx.world_size,
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


def _no_manifest(directory: Path) -> str:
    """The missing-manifest problem, naming the latest complete step directory
    inside ``directory`` when it is a save root rather than a step."""
    steps = sorted(p for p in directory.glob("step_*") if (p / MANIFEST).is_file()) if directory.is_dir() else []
    if steps:
        return f"no manifest.pt here; this looks like a save directory, pass a step such as {steps[-1]}"
    return "no manifest.pt: the save did not complete"


def load_checkpoint(directory, model, optimizer, ctx: ParallelContext, *, data=None,
                    map_location="cpu") -> tuple[int, dict]:
    """Validate ``directory`` for this rank, then restore model, optimizer, RNG and
    data position. Returns ``(step, extra)``. Nothing is modified unless every
    check passes."""
    directory = Path(directory)
    problems: list[str] = []
    manifest_path = directory / MANIFEST
    if not manifest_path.is_file():
        _fail(directory, [_no_manifest(directory)])
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


# --------------------------------------------------- reference checkpoints
REFERENCE_FORMAT_VERSION = 1


def _reference_config_problems(saved: dict | None, model) -> list[str]:
    """The reference's model configuration against this model's: every field the
    reference records must match, and the settings the reference fixes (SwiGLU
    width 4 x n_embd, RoPE theta 10000) must hold here too."""
    ours = _model_config(model)
    if saved is None or ours is None:
        return [f"model configuration: checkpoint {saved!r}, this model {ours!r}"]
    problems = [f"model configuration {key}: checkpoint {value!r}, this model {ours.get(key)!r}"
                for key, value in saved.items() if ours.get(key) != value]
    return problems + reference_config_problems(model.config)


def _adamw_problems(state: dict, model, optimizer) -> list[str]:
    groups = state.get("param_groups") or []
    if len(groups) != 1:
        return [f"optimizer: {len(groups)} parameter groups, one expected"]
    group = groups[0]
    problems = []
    if len(group.get("params", ())) != len(list(model.parameters())):
        problems.append(f"optimizer: {len(group.get('params', ()))} parameters, this model has "
                        f"{len(list(model.parameters()))}")
    if group.get("amsgrad") or group.get("maximize"):
        problems.append("optimizer: amsgrad / maximize AdamW state has no counterpart in FusedAdamW")
    steps = {int(s["step"]) for s in (state.get("state") or {}).values()}
    if len(steps) > 1:
        problems.append(f"optimizer: parameters at different step counts {sorted(steps)}")
    if not hasattr(optimizer, "exp_avg") or not hasattr(optimizer, "flat"):
        problems.append("optimizer: a reference AdamW state loads into FusedAdamW only")
    return problems


def _load_adamw(state: dict, model, optimizer) -> None:
    """torch.optim.AdamW moments, per parameter in ``model.parameters()`` order,
    into FusedAdamW's flat moments: each parameter's moments go to the same
    strided place in the flat moment buffers as its values in the flat
    parameter buffer."""
    group = state["param_groups"][0]
    per_param = state.get("state") or {}
    base = optimizer.flat.data.storage_offset()
    optimizer.exp_avg.zero_()
    optimizer.exp_avg_sq.zero_()
    for index, p in zip(group["params"], model.parameters()):
        entry = per_param.get(index)
        if entry is None:
            continue
        offset = p.data.storage_offset() - base
        for flat, key in ((optimizer.exp_avg, "exp_avg"), (optimizer.exp_avg_sq, "exp_avg_sq")):
            torch.as_strided(flat, p.shape, p.stride(), offset).copy_(entry[key])
    steps = {int(s["step"]) for s in per_param.values()}
    optimizer.step_count = steps.pop() if steps else 0
    optimizer.param_groups = [dict(lr=group["lr"], betas=tuple(group["betas"]), eps=group["eps"],
                                   weight_decay=group["weight_decay"])]


def import_reference_checkpoint(directory, model, optimizer, ctx: ParallelContext, *, data=None,
                                map_location="cpu") -> tuple[int, dict]:
    """Resume from a step directory written by the reference's ``save_checkpoint``
    (``nano_megatron/checkpoint.py:70-126``): the same file layout, a
    ``torch.optim.AdamW`` state, the reference's generator and token-stream
    states. Checks the manifest, this rank's topology, the model configuration
    and the optimizer state first and reports every problem in one
    :class:`CheckpointError`; then loads the model, places the AdamW moments
    into ``optimizer`` (a :class:`~nano_megatron_b200.optim.FusedAdamW`),
    restores the generators and the stream position. Returns ``(step, extra)``
    like :func:`load_checkpoint`; the next save writes this implementation's
    format."""
    directory = Path(directory)
    problems: list[str] = []
    if not (directory / MANIFEST).is_file():
        _fail(directory, [_no_manifest(directory)])
    manifest = _read(directory / MANIFEST, "manifest", "cpu", problems)
    if manifest is None:
        _fail(directory, problems)
    table = [("format version", manifest.get("version"), REFERENCE_FORMAT_VERSION),
             ("world size", manifest.get("world_size"), ctx.world_size),
             ("parallel sizes", manifest.get("parallel_sizes"), _sizes(ctx))]
    problems += [f"{name}: checkpoint {saved!r}, this run {now!r}" for name, saved, now in table if saved != now]
    missing = [n for n in manifest.get("shards") or () if not (directory / n).is_file()]
    if missing:
        problems.append(f"listed shards missing on disk: {missing}")
    if problems:
        _fail(directory, problems)
    shard = _read(directory / shard_name(ctx.rank), "shard", map_location, problems)
    if shard is None:
        _fail(directory, problems)
    table = [("shard format version", shard.get("version"), REFERENCE_FORMAT_VERSION),
             ("rank topology", shard.get("topology"), topology(ctx)),
             ("step (shard vs manifest)", shard.get("step"), manifest.get("step"))]
    problems += [f"{name}: checkpoint {saved!r}, expected {now!r}" for name, saved, now in table if saved != now]
    problems += _reference_config_problems(shard.get("model_config"), model)
    problems += _adamw_problems(shard.get("optimizer") or {}, model, optimizer)
    stream = shard.get("data")
    if stream is not None and data is None:
        problems.append("the shard holds a data-stream position but no stream was passed")
    rng = shard.get("rng") or {}
    if "cuda" in rng and not torch.cuda.is_available():
        problems.append("the shard holds CUDA generator states but CUDA is not available")
    if problems:
        _fail(directory, problems)

    model.load_state_dict(shard["model"])
    _load_adamw(shard["optimizer"], model, optimizer)
    if stream is not None:
        identity = stream.get("identity") or {}
        data.load_state_dict({
            "cursor": stream.get("cursor"),
            "layout": {key: stream.get(key) for key in ("dtype", "seq_len", "dp_rank", "dp_size")},
            "file": {"path": identity.get("path"), "bytes": identity.get("size_bytes"),
                     "mtime_ns": identity.get("mtime_ns")},
        })
    states = {"cpu": rng["torch"], "python": rng["python"]}
    if "cuda" in rng:
        states["cuda"] = rng["cuda"]
    _apply_random_states(states)
    return shard["step"], shard.get("extra") or {}


# GPTConfig fields this implementation adds; the reference's model configuration is the rest
_EXTENSION_FIELDS = ("ffn_hidden_size", "rope_theta", "init_std")


def reference_config_problems(config) -> list[str]:
    """Why the reference could not describe a model of ``config`` (empty when
    it can): its models fix the SwiGLU width at 4 x n_embd and RoPE theta at
    10000."""
    problems = []
    if config.ffn_size != 4 * config.n_embd:
        problems.append(f"SwiGLU width {config.ffn_size}: the reference's models use 4 x n_embd = "
                        f"{4 * config.n_embd}")
    if config.rope_theta != 10000.0:
        problems.append(f"RoPE theta {config.rope_theta}: the reference's models use 10000")
    return problems


def _adamw_state_dict(model, optimizer) -> dict:
    """FusedAdamW's flat moments as a ``torch.optim.AdamW`` state dict over
    ``model.parameters()`` (the inverse of :func:`_load_adamw`): each
    parameter's moments are read from the place its values occupy in the flat
    parameter buffer; the group carries torch's own AdamW defaults."""
    group = optimizer.param_groups[0]
    template = torch.optim.AdamW([torch.zeros(1)], lr=group["lr"], betas=tuple(group["betas"]),
                                 eps=group["eps"], weight_decay=group["weight_decay"])
    params = list(model.parameters())
    saved_group = {k: v for k, v in template.state_dict()["param_groups"][0].items() if k != "params"}
    saved_group["params"] = list(range(len(params)))
    state = {}
    if optimizer.step_count > 0:
        base = optimizer.flat.data.storage_offset()
        for index, p in enumerate(params):
            offset = p.data.storage_offset() - base
            exp_avg, exp_avg_sq = (torch.as_strided(flat, p.shape, p.stride(), offset).detach().to("cpu", copy=True)
                                   for flat in (optimizer.exp_avg, optimizer.exp_avg_sq))
            state[index] = {"step": torch.tensor(float(optimizer.step_count), dtype=torch.float32),
                            "exp_avg": exp_avg, "exp_avg_sq": exp_avg_sq}
    return {"state": state, "param_groups": [saved_group]}


def export_reference_checkpoint(directory, model, optimizer, ctx: ParallelContext, *, step: int,
                                data=None, extra: dict | None = None) -> Path:
    """Save a step directory that the reference's ``load_checkpoint``
    (``nano_megatron/checkpoint.py:129-196``) resumes: the reference's model
    configuration fields, a ``torch.optim.AdamW`` state made from the
    FusedAdamW moments, its generator and token-stream state formats, and the
    same file layout. Refuses, before writing anything, a model the reference
    cannot describe (a SwiGLU width other than 4 x n_embd, RoPE theta other
    than 10000) and an optimizer other than FusedAdamW. Collective like
    :func:`save_checkpoint`; returns this rank's shard path."""
    if not _valid_step(step):
        raise ValueError(f"export_reference_checkpoint: step {step!r} is not a non-negative int")
    config = getattr(model, "config", None)
    problems = ["the model has no GPTConfig"] if config is None else reference_config_problems(config)
    if not hasattr(optimizer, "exp_avg") or not hasattr(optimizer, "flat"):
        problems.append("optimizer: only a FusedAdamW state converts to torch AdamW")
    if problems:
        raise CheckpointError(f"cannot write {directory} for the reference:\n  - " + "\n  - ".join(problems))
    model_config = {k: v for k, v in asdict(config).items() if k not in _EXTENSION_FIELDS}

    def make_shard():
        stream = None
        if data is not None:
            state = data.state_dict()
            stream = {"cursor": state["cursor"], **state["layout"],
                      "identity": {"path": state["file"]["path"], "size_bytes": state["file"]["bytes"],
                                   "mtime_ns": state["file"]["mtime_ns"]}}
        states = _random_states()
        rng = {"torch": states["cpu"], "python": states["python"]}
        if "cuda" in states:
            rng["cuda"] = states["cuda"]
        return {"version": REFERENCE_FORMAT_VERSION, "topology": topology(ctx),
                "model": _host_copy(model.state_dict()), "model_config": model_config,
                "optimizer": _adamw_state_dict(model, optimizer), "step": step, "rng": rng,
                "data": stream, "extra": dict(extra or {})}

    return _write_step(Path(directory), ctx, step, REFERENCE_FORMAT_VERSION, make_shard)
