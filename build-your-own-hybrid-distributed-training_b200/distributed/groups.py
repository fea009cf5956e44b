"""Process-group registry: the only place that calls ``dist.new_group``.

Every rank must call ``new_group`` for every group, in the same order, even for
groups it is not a member of; a rank that skipped one would desynchronise the
NCCL communicator ids.  The registry therefore walks ``GROUP_CREATION_ORDER``
and, inside each dimension, ``ParallelTopology.all_group_rank_lists`` (sorted by
first member).  Single-member groups get no communicator (``GroupHandle.trivial``
semantics), identical rank lists share one communicator, and teardown runs in
reverse order.  Same contract as ``src/hybrid_training/distributed/groups.py:69-428``.
"""

from __future__ import annotations

from dataclasses import dataclass
from datetime import timedelta
from typing import Any

import torch.distributed as dist

from ..errors import CollectiveError, DistributedInitializationError, format_error
from ..logging import get_logger
from .topology import COMPOSITE_GROUPS, DIMENSIONS, ParallelTopology

__all__ = ["GROUP_CREATION_ORDER", "GroupHandle", "ProcessGroupRegistry", "known_group_names", "validate_group_membership"]

_LOG = get_logger(__name__)

GROUP_CREATION_ORDER: tuple[str, ...] = ("data_parallel", "shard", "sequence", "tensor", "dp_shard", "tensor_sequence")


@dataclass(frozen=True)
class GroupHandle:
    """This rank's view of one process group.

    ``process_group`` is ``None`` for single-member groups; every collective
    wrapper short-circuits those, so single-process code runs unmodified.
    """

    name: str
    ranks: tuple[int, ...]
    local_rank: int
    global_rank: int
    process_group: Any

    @property
    def size(self) -> int:
        return len(self.ranks)

    @property
    def is_trivial(self) -> bool:
        return len(self.ranks) == 1

    @property
    def source_rank(self) -> int:
        return self.ranks[0]

    @classmethod
    def trivial(cls, name: str = "trivial", rank: int = 0) -> GroupHandle:
        """A one-member group with no communicator (the test fake backend)."""
        return cls(name=name, ranks=(rank,), local_rank=0, global_rank=rank, process_group=None)

    def __repr__(self) -> str:
        return f"GroupHandle(name={self.name!r}, size={self.size}, local_rank={self.local_rank}, ranks={self.ranks})"


class ProcessGroupRegistry:
    """Creates and owns every sub-group of the 4-D grid."""

    def __init__(self, topology: ParallelTopology, rank: int, *, timeout: timedelta | None = None,
                 backend: str | None = None, create: bool = True) -> None:
        if create and not dist.is_initialized():
            raise DistributedInitializationError(format_error(
                "groups.ProcessGroupRegistry", "sub-groups are built from the world process group, which does not exist yet",
                rank=rank, world_size=topology.world_size, resolution="call init_distributed() first"))
        self._topology = topology
        self._rank = rank
        self._handles: dict[str, GroupHandle] = {}
        self._created: list[tuple[str, tuple[int, ...]]] = []
        self._destroyed = False
        world = tuple(range(topology.world_size))
        default = dist.group.WORLD if create else None
        communicators: dict[tuple[int, ...], Any] = {world: default} if create else {}
        kwargs: dict[str, Any] = {}
        if timeout is not None:
            kwargs["timeout"] = timeout
        if backend is not None:
            kwargs["backend"] = backend
        for name in GROUP_CREATION_ORDER:
            mine: tuple[tuple[int, ...], Any] | None = None
            for members in topology.all_group_rank_lists(name):
                self._created.append((name, members))
                pg = None
                if create and len(members) > 1:
                    if members not in communicators:
                        communicators[members] = dist.new_group(ranks=list(members), **kwargs)
                    pg = communicators[members]
                if rank in members:
                    mine = (members, pg)
            if mine is None:
                raise DistributedInitializationError(format_error(
                    "groups.ProcessGroupRegistry", f"this rank is in none of the {name!r} group", rank=rank,
                    world_size=topology.world_size, resolution="the rank grid arithmetic is inconsistent (an internal error)"))
            self._handles[name] = GroupHandle(name, mine[0], mine[0].index(rank), rank, mine[1])
        self._handles["world"] = GroupHandle("world", world, rank, rank, default)
        _LOG.debug("%d communicators created", len(self._created))

    def get(self, name: str) -> GroupHandle:
        if self._destroyed:
            raise CollectiveError(format_error("groups.get", "the group registry was already torn down",
                                               rank=self._rank, world_size=self._topology.world_size,
                                               resolution="keep using groups only while their context is active"))
        if name == "sequence_effective":
            name = self._topology.sequence_group_name
        handle = self._handles.get(name)
        if handle is None:
            raise CollectiveError(format_error("groups.get", "no group is registered under this name", rank=self._rank,
                                               world_size=self._topology.world_size,
                                               expected=[*sorted(self._handles), "sequence_effective"], observed=name,
                                               resolution="ask for one of the group names the registry lists"))
        return handle

    def __getitem__(self, name: str) -> GroupHandle:
        return self.get(name)

    def __contains__(self, name: str) -> bool:
        return name in self._handles or name == "sequence_effective"

    @property
    def names(self) -> tuple[str, ...]:
        return (*GROUP_CREATION_ORDER, "world")

    @property
    def creation_log(self) -> tuple[tuple[str, tuple[int, ...]], ...]:
        """Every ``(dimension, members)`` visited, in creation order (identical on all ranks)."""
        return tuple(self._created)

    def describe(self) -> str:
        lines = [f"communicators of rank {self._rank}:"]
        for name in self.names:
            h = self._handles[name]
            lines.append(f"  {name:<16} size={h.size:<3} local_rank={h.local_rank:<3} ranks={h.ranks}")
        return "\n".join(lines)

    def destroy(self) -> None:
        """Destroy sub-group communicators in reverse creation order (never the default group)."""
        if self._destroyed:
            return
        self._destroyed = True
        default = dist.group.WORLD if dist.is_initialized() else None
        done: set[int] = set()
        for name in reversed(self.names):
            handle = self._handles.get(name)
            if handle is None or handle.process_group is None or handle.process_group is default:
                continue
            if id(handle.process_group) in done:
                continue
            done.add(id(handle.process_group))
            dist.destroy_process_group(handle.process_group)
        self._handles.clear()


def validate_group_membership(handle: GroupHandle, rank: int, operation: str) -> None:
    if rank not in handle.ranks:
        raise CollectiveError(format_error(operation, f"this rank does not belong to group {handle.name!r}", rank=rank,
                                           expected=f"rank in {handle.ranks}", observed=rank,
                                           resolution="pass the group handle this rank obtained from the registry"))


def known_group_names() -> tuple[str, ...]:
    return (*DIMENSIONS, *COMPOSITE_GROUPS, "sequence_effective")
