"""Per-rank view of the TP x PP x DP process grid.

Ranks are laid out as ``rank = (pp * dp_size + dp) * tp_size + tp``: tensor
parallelism varies fastest so that a TP group is a block of consecutive ranks
(one NVSwitch-local set of GPUs on a node), then data parallelism, then pipeline
stages. Every rank creates every subgroup in the same order because
``torch.distributed.new_group`` is a collective over the whole world.

Parity: ``nano_megatron/parallel.py:11-143`` (grid order, group semantics,
tied first/last-stage group, stage predicates and neighbour lookup).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch.distributed as dist


@dataclass(frozen=True)
class ParallelContext:
    """Topology of one rank. Immutable; passed explicitly, never global.
    Parity: ``nano_megatron/parallel.py:11-72`` (same fields; ``resources``
    is added for per-group state such as symmetric workspaces)."""

    rank: int
    world_size: int
    tp_size: int
    tp_rank: int
    pp_size: int
    pp_rank: int
    dp_size: int
    dp_rank: int
    tp_group: dist.ProcessGroup | None = None
    pp_group: dist.ProcessGroup | None = None
    dp_group: dist.ProcessGroup | None = None
    tied_group: dist.ProcessGroup | None = None
    tp_ranks: tuple[int, ...] = (0,)
    pp_ranks: tuple[int, ...] = (0,)
    dp_ranks: tuple[int, ...] = (0,)
    # Lazily created per-group resources (symmetric buffers, comm streams).
    # Excluded from equality so two contexts with equal topology compare equal.
    resources: dict = field(default_factory=dict, compare=False, repr=False)

    @classmethod
    def single(cls) -> "ParallelContext":
        """A one-rank context: no groups, every size 1."""
        return cls(rank=0, world_size=1, tp_size=1, tp_rank=0, pp_size=1,
                   pp_rank=0, dp_size=1, dp_rank=0)

    @property
    def is_first_stage(self) -> bool:
        return self.pp_rank == 0

    @property
    def is_last_stage(self) -> bool:
        return self.pp_rank == self.pp_size - 1

    @property
    def previous_pipeline_rank(self) -> int:
        if self.is_first_stage:
            raise RuntimeError(f"pipeline stage {self.pp_rank} is the first one; nothing sends to it")
        return self.pp_ranks[self.pp_rank - 1]

    @property
    def next_pipeline_rank(self) -> int:
        if self.is_last_stage:
            raise RuntimeError(f"pipeline stage {self.pp_rank} is the last of {self.pp_size}; it sends to nobody")
        return self.pp_ranks[self.pp_rank + 1]

    def describe(self) -> str:
        """One line per rank: grid coordinate and the members of its groups."""
        coord = f"(pp={self.pp_rank}, dp={self.dp_rank}, tp={self.tp_rank})"
        shape = f"{self.pp_size}x{self.dp_size}x{self.tp_size}"
        return (f"[rank {self.rank} of {self.world_size}] grid {shape} at {coord}; "
                f"TP peers {list(self.tp_ranks)}, PP chain {list(self.pp_ranks)}, "
                f"DP replicas {list(self.dp_ranks)}")


def grid_ranks(world_size: int, tp_size: int, pp_size: int):
    """Return the nested rank lists ``grid[pp][dp][tp]`` for a world size."""
    if tp_size <= 0 or pp_size <= 0:
        raise ValueError(f"tensor ({tp_size}) and pipeline ({pp_size}) widths must both be >= 1")
    if world_size % (tp_size * pp_size):
        raise ValueError(f"{world_size} ranks cannot be split into TP {tp_size} x PP {pp_size} "
                         f"blocks ({world_size} % {tp_size * pp_size} != 0)")
    dp_size = world_size // (tp_size * pp_size)
    return [[[(p * dp_size + d) * tp_size + t for t in range(tp_size)]
             for d in range(dp_size)] for p in range(pp_size)], dp_size


def init_parallel(tp_size: int = 1, pp_size: int = 1) -> ParallelContext:
    """Create all TP, DP, PP and tied-embedding groups; return this rank's view.
    Parity: ``nano_megatron/parallel.py:75-143`` (grid order and group creation
    order)."""
    if not dist.is_initialized():
        raise RuntimeError("init_parallel builds groups over an existing world: call "
                           "torch.distributed.init_process_group first")
    world_size = dist.get_world_size()
    rank = dist.get_rank()
    grid, dp_size = grid_ranks(world_size, tp_size, pp_size)

    found: dict[str, tuple] = {}

    def make(kind: str, ranks: list[int]) -> None:
        group = dist.new_group(ranks)
        if rank in ranks:
            found[kind] = (group, tuple(ranks))

    for p in range(pp_size):
        for d in range(dp_size):
            make("tp", grid[p][d])
    for p in range(pp_size):
        for t in range(tp_size):
            make("dp", [grid[p][d][t] for d in range(dp_size)])
    for d in range(dp_size):
        for t in range(tp_size):
            column = [grid[p][d][t] for p in range(pp_size)]
            make("pp", column)
            if pp_size > 1:
                make("tied", [column[0], column[-1]])

    tp_group, tp_ranks = found["tp"]
    dp_group, dp_ranks = found["dp"]
    pp_group, pp_ranks = found["pp"]
    tied_group = found["tied"][0] if "tied" in found else None
    return ParallelContext(
        rank=rank, world_size=world_size,
        tp_size=tp_size, tp_rank=tp_ranks.index(rank),
        pp_size=pp_size, pp_rank=pp_ranks.index(rank),
        dp_size=dp_size, dp_rank=dp_ranks.index(rank),
        tp_group=tp_group, pp_group=pp_group, dp_group=dp_group, tied_group=tied_group,
        tp_ranks=tp_ranks, pp_ranks=pp_ranks, dp_ranks=dp_ranks,
    )
