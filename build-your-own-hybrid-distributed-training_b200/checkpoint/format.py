"""Checkpoint naming, versioning, path safety and file digests.

The on-disk names are fixed by the format (reference
``src/hybrid_training/checkpoint/format.py:64-292``) so checkpoints written by
either implementation are laid out the same way:
``checkpoint-step-NNNNNN/`` containing ``manifest.json``, ``metadata.json`` and
``rank-NNNNN.pt``; a write is staged in ``.staging-<final>-<token>`` and
renamed into place.  A manifest may only name files matching ``rank-NNNNN.pt``
that resolve inside the checkpoint directory.
"""

from __future__ import annotations

import hashlib
import re
from pathlib import Path

from ..errors import CheckpointError, CheckpointVersionError, format_error

__all__ = [
    "CHECKPOINT_DIRECTORY_PATTERN",
    "CURRENT_FORMAT_VERSION",
    "MANIFEST_FILENAME",
    "METADATA_FILENAME",
    "SUPPORTED_FORMAT_VERSIONS",
    "checkpoint_directory_name",
    "file_digest",
    "resolve_inside",
    "shard_filename",
    "staging_directory_name",
    "step_from_directory_name",
    "validate_format_version",
    "validate_shard_filename",
]

CURRENT_FORMAT_VERSION = "1.0"
SUPPORTED_FORMAT_VERSIONS = frozenset({"1.0"})
MANIFEST_FILENAME = "manifest.json"
METADATA_FILENAME = "metadata.json"
CHECKPOINT_DIRECTORY_PATTERN = re.compile(r"^checkpoint-step-(\d{6,})$")
_SHARD_PATTERN = re.compile(r"^rank-(\d{5,})\.pt$")
_STAGING_PREFIX = ".staging-"


def checkpoint_directory_name(step: int) -> str:
    if step < 0:
        raise CheckpointError(format_error("checkpoint.directory_name", "checkpoint steps start at 0", expected=">= 0",
                                           observed=step, resolution="give the optimizer step the checkpoint belongs to"))
    return f"checkpoint-step-{step:06d}"


def step_from_directory_name(name: str) -> int | None:
    m = CHECKPOINT_DIRECTORY_PATTERN.match(name)
    return int(m.group(1)) if m else None


def staging_directory_name(final_name: str, token: str) -> str:
    return f"{_STAGING_PREFIX}{final_name}-{token}"


def shard_filename(rank: int) -> str:
    if rank < 0:
        raise CheckpointError(format_error("checkpoint.shard_filename", "a global rank cannot be negative", expected=">= 0",
                                           observed=rank, resolution="pass a global rank"))
    return f"rank-{rank:05d}.pt"


def validate_shard_filename(name: str) -> str:
    if not _SHARD_PATTERN.match(name):
        raise CheckpointError(format_error(
            "checkpoint.validate_shard_filename", "the manifest names a file outside the shard naming rule; refusing it, "
            "because a manifest must never point the reader at an arbitrary path", expected="rank-NNNNN.pt", observed=name,
            resolution="the manifest was edited by hand or damaged; do not load it"))
    return name


def resolve_inside(root: Path, name: str) -> Path:
    base = root.resolve()
    candidate = (base / name).resolve()
    try:
        candidate.relative_to(base)
    except ValueError as exc:
        raise CheckpointError(format_error("checkpoint.resolve_inside", "after resolving links the file lies outside the checkpoint directory",
                                           expected=f"a path under {base}", observed=str(candidate),
                                           resolution="keep every payload file inside the checkpoint directory (no links pointing out)")) from exc
    return candidate


def file_digest(path: Path, *, chunk_size: int = 1 << 22) -> str:
    """Streaming SHA-256 of a file."""
    h = hashlib.sha256()
    try:
        with path.open("rb") as f:
            for chunk in iter(lambda: f.read(chunk_size), b""):
                h.update(chunk)
    except OSError as exc:
        raise CheckpointError(format_error("checkpoint.file_digest", "reading a checkpoint file failed", expected="a readable file",
                                           observed=f"{path}: {exc}", resolution="check permissions and that the file exists")) from exc
    return h.hexdigest()


def validate_format_version(version: str) -> str:
    if version not in SUPPORTED_FORMAT_VERSIONS:
        raise CheckpointVersionError(format_error("checkpoint.validate_format_version", "this reader does not know the checkpoint's format version",
                                                  expected=sorted(SUPPORTED_FORMAT_VERSIONS), observed=version,
                                                  resolution="use the package version that wrote the checkpoint"))
    return version
