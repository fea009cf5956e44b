"""The 4-D rank grid: pure arithmetic, no communication.

A rank is a mixed-radix number over ``(data_parallel, shard, sequence, tensor)``
with ``tensor`` the fastest-varying digit::

    rank = ((dp * S + sh) * Q + sq) * T + tp

so the members of a tensor group are consecutive ranks, which on one NVSwitch
node means consecutive GPUs.  Composite groups combine dimensions:
``dp_shard`` (data_parallel x shard, the group that sees different batches),
``tensor_sequence`` (sequence x tensor, the group that sees the same batch) and
``world``.  Same conventions as ``src/hybrid_training/distributed/topology.py:83-494``.
"""

from __future__ import annotations

import itertools
from collections.abc import Iterable
from dataclasses import dataclass

from ..config import SequenceParallelMode, TopologyConfig
from ..errors import TopologyError, format_error

__all__ = ["COMPOSITE_GROUPS", "DIMENSIONS", "ParallelTopology", "RankCoordinates"]

DIMENSIONS: tuple[str, ...] = ("data_parallel", "shard", "sequence", "tensor")
COMPOSITE_GROUPS: dict[str, tuple[str, ...]] = {
    "dp_shard": ("data_parallel", "shard"),
    "tensor_sequence": ("sequence", "tensor"),
    "world": DIMENSIONS,
}


@dataclass(frozen=True)
class RankCoordinates:
    data_parallel: int
    shard: int
    sequence: int
    tensor: int

    def as_tuple(self) -> tuple[int, int, int, int]:
        return (self.data_parallel, self.shard, self.sequence, self.tensor)

    def __getitem__(self, dimension: str) -> int:
        if dimension not in DIMENSIONS:
            raise KeyError(f"{dimension!r} is not a grid dimension (the grid has {', '.join(DIMENSIONS)})")
        return int(getattr(self, dimension))

    def label(self) -> str:
        return f"dp{self.data_parallel}/sh{self.shard}/sq{self.sequence}/tp{self.tensor}"


class ParallelTopology:
    """Rank <-> coordinate mapping and group enumeration for one world size."""

    def __init__(self, config: TopologyConfig, world_size: int) -> None:
        config.validate_against_world_size(world_size)
        self._config = config
        self._world_size = world_size
        self._sizes = {
            "data_parallel": config.data_parallel_size,
            "shard": config.shard_parallel_size,
            "sequence": config.sequence_parallel_size,
            "tensor": config.tensor_parallel_size,
        }
        # Place value of each digit: tensor = 1, sequence = T, shard = Q*T, dp = S*Q*T.
        self._place: dict[str, int] = {}
        place = 1
        for dim in reversed(DIMENSIONS):
            self._place[dim] = place
            place *= self._sizes[dim]

    @property
    def config(self) -> TopologyConfig:
        return self._config

    @property
    def world_size(self) -> int:
        return self._world_size

    @property
    def sizes(self) -> dict[str, int]:
        return dict(self._sizes)

    def size(self, dimension: str) -> int:
        out = 1
        for dim in self._resolve(dimension):
            out *= self._sizes[dim]
        return out

    def coordinates_of(self, rank: int) -> RankCoordinates:
        self._check_rank(rank)
        digits = {dim: (rank // self._place[dim]) % self._sizes[dim] for dim in DIMENSIONS}
        return RankCoordinates(**digits)

    def rank_of(self, coordinates: RankCoordinates | Iterable[int]) -> int:
        values = coordinates.as_tuple() if isinstance(coordinates, RankCoordinates) else tuple(coordinates)
        if len(values) != len(DIMENSIONS):
            raise TopologyError(format_error("topology.rank_of", "the coordinate tuple has the wrong length", expected=len(DIMENSIONS),
                                             observed=len(values), resolution=f"give exactly one index per grid dimension {DIMENSIONS}"))
        rank = 0
        for dim, value in zip(DIMENSIONS, values):
            if not 0 <= value < self._sizes[dim]:
                raise TopologyError(format_error("topology.rank_of", f"the index along {dim!r} is out of range",
                                                 expected=f"0 <= c < {self._sizes[dim]}", observed=value,
                                                 resolution="each index has to be below the size of its dimension"))
            rank += value * self._place[dim]
        return rank

    def _members(self, varying: tuple[str, ...], fixed: RankCoordinates | dict[str, int]) -> tuple[int, ...]:
        axes = [range(self._sizes[d]) if d in varying else (fixed[d],) for d in DIMENSIONS]
        return tuple(sorted(self.rank_of(c) for c in itertools.product(*axes)))

    def group_ranks(self, dimension: str, rank: int) -> tuple[int, ...]:
        """Members (sorted global ranks) of ``rank``'s group along ``dimension``."""
        self._check_rank(rank)
        return self._members(self._resolve(dimension), self.coordinates_of(rank))

    def all_group_rank_lists(self, dimension: str) -> tuple[tuple[int, ...], ...]:
        """Every group along ``dimension``, ordered by first member (the creation order)."""
        varying = self._resolve(dimension)
        fixed_dims = [d for d in DIMENSIONS if d not in varying]
        groups = []
        for values in itertools.product(*(range(self._sizes[d]) for d in fixed_dims)):
            groups.append(self._members(varying, dict(zip(fixed_dims, values))))
        return tuple(sorted(groups, key=lambda g: g[0]))

    def local_rank_in_group(self, dimension: str, rank: int) -> int:
        return self.group_ranks(dimension, rank).index(rank)

    def group_source_rank(self, dimension: str, rank: int) -> int:
        return self.group_ranks(dimension, rank)[0]

    def neighbour_ranks(self, dimension: str, rank: int) -> tuple[int, int]:
        """(previous, next) rank of a ring over the group; used by ring attention."""
        members = self.group_ranks(dimension, rank)
        i = members.index(rank)
        return members[(i - 1) % len(members)], members[(i + 1) % len(members)]

    @property
    def sequence_group_name(self) -> str:
        return "tensor" if self._config.sequence_parallel_mode == SequenceParallelMode.TENSOR_GROUP else "sequence"

    @property
    def sequence_parallel_size(self) -> int:
        return self.size(self.sequence_group_name)

    @property
    def sequence_parallel_enabled(self) -> bool:
        return self._config.sequence_parallel_enabled

    def describe(self, rank: int) -> str:
        coords = self.coordinates_of(rank)
        lines = [
            f"rank {rank}/{self._world_size}  coordinates {coords.label()}",
            "  sizes: " + ", ".join(f"{d}={self._sizes[d]}" for d in DIMENSIONS),
            f"  sequence split       : {self._config.sequence_parallel_mode} (effective size {self.sequence_parallel_size})",
        ]
        for name in (*DIMENSIONS, *COMPOSITE_GROUPS):
            members = self.group_ranks(name, rank)
            lines.append(f"  {name:<16} size={len(members):<3} local_rank={members.index(rank):<3} members={members}")
        return "\n".join(lines)

    def summary(self) -> dict[str, object]:
        """JSON-safe description recorded in checkpoint manifests."""
        return {
            "world_size": self._world_size,
            "sizes": dict(self._sizes),
            "sequence_parallel_mode": self._config.sequence_parallel_mode,
            "dimension_order": list(DIMENSIONS),
        }

    def _resolve(self, dimension: str) -> tuple[str, ...]:
        if dimension in DIMENSIONS:
            return (dimension,)
        if dimension in COMPOSITE_GROUPS:
            return COMPOSITE_GROUPS[dimension]
        raise TopologyError(format_error("topology.resolve", "not a grid dimension nor a composite group",
                                         expected=sorted({*DIMENSIONS, *COMPOSITE_GROUPS}), observed=dimension,
                                         resolution="ask for a dimension or one of the composite groups"))

    def _check_rank(self, rank: int) -> None:
        if not 0 <= rank < self._world_size:
            raise TopologyError(format_error("topology.check_rank", "the rank is not in this grid", world_size=self._world_size,
                                             expected=f"0 <= rank < {self._world_size}", observed=rank,
                                             resolution="this grid was laid out for another number of ranks"))

    def __repr__(self) -> str:
        return f"ParallelTopology(world_size={self._world_size}, " + ", ".join(f"{d}={self._sizes[d]}" for d in DIMENSIONS) + ")"
