"""Exception hierarchy and the rank-aware error message format.

Every error raised by the framework carries five parts so that a log line from
one rank of a 4-D grid is self-explanatory::

    [rank R/W] operation: problem; expected X, observed Y. Fix: what to do

The hierarchy mirrors the reference (``src/hybrid_training/errors.py:45-197``):
``ConfigurationError`` is also a ``ValueError`` and ``UnsupportedFeatureError``
is also a ``NotImplementedError`` so generic handlers keep working.
``KernelError`` is new: it is raised when a native kernel reports a failure
status (for example a bounded device-side wait that expired).
"""

from __future__ import annotations

from typing import Any

__all__ = [
    "CheckpointCorruptionError",
    "CheckpointError",
    "CheckpointTopologyError",
    "CheckpointVersionError",
    "CollectiveError",
    "ConfigurationError",
    "DistributedInitializationError",
    "HybridTrainingError",
    "IncompleteCheckpointError",
    "KernelError",
    "ParameterConsistencyError",
    "ShardingError",
    "TensorParallelError",
    "TopologyError",
    "UnsupportedFeatureError",
    "format_error",
]


def format_error(
    operation: str,
    problem: str,
    *,
    rank: int | None = None,
    world_size: int | None = None,
    expected: Any = None,
    observed: Any = None,
    resolution: str | None = None,
) -> str:
    """Build the five-part message used by every exception in the package."""
    if rank is not None and world_size is not None:
        head = f"[rank {rank}/{world_size}] "
    elif rank is not None:
        head = f"[rank {rank}] "
    else:
        head = ""
    parts = [f"{head}{operation}: {problem}"]
    if expected is not None or observed is not None:
        parts.append(f"; expected {expected!r}, observed {observed!r}")
    if resolution:
        parts.append(f". Fix: {resolution}")
    return "".join(parts)


class HybridTrainingError(Exception):
    """Root of every error raised by this package."""


class ConfigurationError(HybridTrainingError, ValueError):
    """An illegal configuration value, detected at construction time."""


class DistributedInitializationError(HybridTrainingError):
    """The process group, device or launch environment could not be set up."""


class TopologyError(ConfigurationError):
    """The 4-D rank grid does not factor the world size or is inconsistent."""


class CollectiveError(HybridTrainingError):
    """A collective was called with bad arguments or failed on some rank."""


class ParameterConsistencyError(HybridTrainingError):
    """Ranks that must agree (structure, layout, values) do not."""


class ShardingError(HybridTrainingError):
    """Flat-parameter, bucket or shard bookkeeping is inconsistent."""


class TensorParallelError(HybridTrainingError):
    """A tensor-parallel layer was configured with incompatible shapes."""


class UnsupportedFeatureError(HybridTrainingError, NotImplementedError):
    """A feature combination that is deliberately not supported."""


class KernelError(HybridTrainingError):
    """A native kernel returned a failure status (e.g. a device wait timed out)."""


class CheckpointError(HybridTrainingError):
    """Base class for checkpoint failures."""


class IncompleteCheckpointError(CheckpointError):
    """The checkpoint is missing files, shards or the completion marker."""


class CheckpointCorruptionError(CheckpointError):
    """A file's size, checksum or contents disagree with the manifest."""


class CheckpointVersionError(CheckpointError):
    """The on-disk format version is not supported by this reader."""


class CheckpointTopologyError(CheckpointError):
    """The checkpoint cannot be loaded at the current topology."""
