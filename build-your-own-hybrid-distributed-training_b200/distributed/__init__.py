"""Distributed runtime: grid arithmetic, process groups, context, collectives, launcher, peer memory.

Import order is acyclic: ``topology -> groups -> context -> collectives ->
launch``; ``symmetric`` (peer-mapped workspaces for in-kernel collectives) is
created lazily by the context.
"""

from .collectives import (
    AsyncWork,
    CommunicationRecorder,
    CommunicationStats,
    ReduceOp,
    all_gather_object_in_group,
    all_gather_tensor,
    all_reduce,
    all_to_all_tensor,
    assert_metadata_consistent,
    assert_tensor_consistent,
    broadcast,
    concat_shard_sizes,
    recv_tensor,
    reduce_scatter_tensor,
    send_tensor,
    sum_scalar,
    wait_all,
)
from .context import (
    DistributedContext,
    LaunchEnvironment,
    current_context,
    distributed_context,
    find_free_port,
    init_distributed,
    is_context_active,
)
from .groups import GROUP_CREATION_ORDER, GroupHandle, ProcessGroupRegistry
from .launch import WorkerFailure, WorkerResult, launch_workers, torchrun_environment_summary
from .topology import COMPOSITE_GROUPS, DIMENSIONS, ParallelTopology, RankCoordinates

__all__ = [
    "COMPOSITE_GROUPS",
    "DIMENSIONS",
    "GROUP_CREATION_ORDER",
    "AsyncWork",
    "CommunicationRecorder",
    "CommunicationStats",
    "DistributedContext",
    "GroupHandle",
    "LaunchEnvironment",
    "ParallelTopology",
    "ProcessGroupRegistry",
    "RankCoordinates",
    "ReduceOp",
    "WorkerFailure",
    "WorkerResult",
    "all_gather_object_in_group",
    "all_gather_tensor",
    "all_reduce",
    "all_to_all_tensor",
    "assert_metadata_consistent",
    "assert_tensor_consistent",
    "broadcast",
    "concat_shard_sizes",
    "current_context",
    "distributed_context",
    "find_free_port",
    "init_distributed",
    "is_context_active",
    "launch_workers",
    "recv_tensor",
    "reduce_scatter_tensor",
    "send_tensor",
    "sum_scalar",
    "torchrun_environment_summary",
    "wait_all",
]
