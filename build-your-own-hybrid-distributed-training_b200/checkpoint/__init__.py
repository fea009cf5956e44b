"""Manifest-based distributed checkpoints with integrity checks and resharding."""

from .format import (
    CURRENT_FORMAT_VERSION,
    MANIFEST_FILENAME,
    METADATA_FILENAME,
    SUPPORTED_FORMAT_VERSIONS,
    checkpoint_directory_name,
    file_digest,
    shard_filename,
    validate_format_version,
    validate_shard_filename,
)
from .manifest import CheckpointManifest, FileRecord, ShardRecord, TensorRecord
from .reader import LoadedCheckpoint, inspect_checkpoint, load_checkpoint, read_metadata
from .reshard import ShardFileCache, describe_reshard, read_tensor_range, verify_files
from .writer import CheckpointWriteResult, find_latest_checkpoint, prune_checkpoints, save_checkpoint

__all__ = [
    "CURRENT_FORMAT_VERSION",
    "MANIFEST_FILENAME",
    "METADATA_FILENAME",
    "SUPPORTED_FORMAT_VERSIONS",
    "CheckpointManifest",
    "CheckpointWriteResult",
    "FileRecord",
    "LoadedCheckpoint",
    "ShardFileCache",
    "ShardRecord",
    "TensorRecord",
    "checkpoint_directory_name",
    "describe_reshard",
    "file_digest",
    "find_latest_checkpoint",
    "inspect_checkpoint",
    "load_checkpoint",
    "prune_checkpoints",
    "read_metadata",
    "read_tensor_range",
    "save_checkpoint",
    "shard_filename",
    "validate_format_version",
    "validate_shard_filename",
    "verify_files",
]
