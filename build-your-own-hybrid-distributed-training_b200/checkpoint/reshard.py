"""Reading arbitrary global intervals back out of a checkpoint (the resharding core).

``read_tensor_range(record, wanted)`` assembles ``[wanted.start, wanted.end)``
of a tensor's flattened global data from whichever shard files cover it, in
offset order, raising on gaps.  ``ShardFileCache`` loads each payload file at
most once, after checking its size and (optionally) SHA-256 against the
manifest, with ``torch.load(weights_only=True)`` so a payload can never
execute code.  Same contract as ``src/hybrid_training/checkpoint/reshard.py:54-419``.
"""

from __future__ import annotations

from collections.abc import Mapping
from pathlib import Path
from typing import Any

import torch

from ..errors import CheckpointCorruptionError, CheckpointError, IncompleteCheckpointError, format_error
from ..utils.tensors import ShardRange
from .format import file_digest, resolve_inside, validate_shard_filename
from .manifest import CheckpointManifest, TensorRecord

__all__ = ["ShardFileCache", "describe_reshard", "read_tensor_range", "verify_files"]


def _check_file(directory: Path, manifest: CheckpointManifest, name: str, *, verify: bool, where: str) -> Path:
    validate_shard_filename(name)
    path = resolve_inside(directory, name)
    if not path.is_file():
        raise IncompleteCheckpointError(format_error(where, "a payload file named by the manifest is not on disk", expected=name,
                                                     observed="absent", resolution="restore the file or resume from an earlier checkpoint"))
    record = manifest.files.get(name)
    if record is None:
        raise CheckpointCorruptionError(format_error(where, "the manifest has no size/checksum entry for this file",
                                                     expected="a record in the manifest's files table", observed=name,
                                                     resolution="manifest.json is incomplete or was edited"))
    size = path.stat().st_size
    if size != record.bytes:
        raise CheckpointCorruptionError(format_error(where, f"shard file {name!r} has the wrong size (truncated or overwritten)",
                                                     expected=f"{record.bytes} bytes", observed=f"{size} bytes",
                                                     resolution="put the original file back, or use an older checkpoint"))
    if verify:
        digest = file_digest(path)
        if digest != record.sha256:
            raise CheckpointCorruptionError(format_error(where, f"shard file {name!r} has a SHA-256 that differs from the manifest",
                                                         expected=record.sha256, observed=digest,
                                                         resolution="the file is corrupt; restore it or discard the checkpoint"))
    return path


class ShardFileCache:
    def __init__(self, directory: Path, manifest: CheckpointManifest, *, verify_checksums: bool = True) -> None:
        self._directory, self._manifest, self._verify = Path(directory), manifest, verify_checksums
        self._loaded: dict[str, Mapping[str, torch.Tensor]] = {}

    def get(self, filename: str) -> Mapping[str, torch.Tensor]:
        if filename in self._loaded:
            return self._loaded[filename]
        path = _check_file(self._directory, self._manifest, filename, verify=self._verify, where="reshard.ShardFileCache.get")
        try:
            payload = torch.load(path, map_location="cpu", weights_only=True)
        except Exception as exc:
            raise CheckpointCorruptionError(format_error("reshard.ShardFileCache.get", f"shard file {filename!r} could not be loaded with torch.load",
                                                         expected="a dict of tensors written by torch.save", observed=repr(exc),
                                                         resolution="the file is corrupt or not a tensor payload")) from exc
        if not isinstance(payload, dict):
            raise CheckpointCorruptionError(format_error("reshard.ShardFileCache.get", f"shard file {filename!r} does not hold a mapping",
                                                         expected="dict[str, Tensor]", observed=type(payload).__name__,
                                                         resolution="the file was not written by this format"))
        self._loaded[filename] = payload
        return payload

    def clear(self) -> None:
        self._loaded.clear()

    @property
    def loaded_files(self) -> tuple[str, ...]:
        return tuple(sorted(self._loaded))


def read_tensor_range(record: TensorRecord, wanted: ShardRange, cache: ShardFileCache, *, dtype: torch.dtype | None = None) -> torch.Tensor:
    """Elements ``[wanted.start, wanted.end)`` of the flattened global tensor."""
    if wanted.length == 0:
        return torch.empty(0, dtype=dtype or torch.float32)
    if wanted.end > record.numel:
        raise CheckpointError(format_error("reshard.read_tensor_range", f"the wanted interval of {record.key!r} runs past the end",
                                           expected=f"end <= {record.numel}", observed=wanted.end,
                                           resolution="build the same model that was saved"))
    pieces = record.shards_overlapping(wanted)
    if not pieces:
        raise IncompleteCheckpointError(format_error("reshard.read_tensor_range", f"no shard of {record.key!r} covers the range",
                                                     expected=f"a shard overlapping [{wanted.start}, {wanted.end})",
                                                     observed=[(s.offset, s.length) for s in record.shards],
                                                     resolution="some data of the checkpoint is absent"))
    out: torch.Tensor | None = None
    cursor, filled = wanted.start, 0
    for shard, overlap in pieces:
        if overlap.start != cursor:
            raise IncompleteCheckpointError(format_error("reshard.read_tensor_range", f"no shard covers part of {record.key!r}",
                                                         expected=f"a shard beginning at element {cursor}",
                                                         observed=f"the following shard begins at {overlap.start}",
                                                         resolution="a payload file is absent or lost entries"))
        payload = cache.get(shard.file)
        stored = payload.get(shard.key)
        if stored is None:
            raise CheckpointCorruptionError(format_error("reshard.read_tensor_range", f"{shard.file!r} has no entry {shard.key!r}",
                                                         expected=shard.key, observed=sorted(payload)[:8],
                                                         resolution="the manifest and payload disagree; the checkpoint is corrupt"))
        flat = stored.reshape(-1)
        if flat.numel() != shard.length:
            raise CheckpointCorruptionError(format_error("reshard.read_tensor_range", f"shard {shard.key!r} length differs from its record",
                                                         expected=shard.length, observed=flat.numel(),
                                                         resolution="the manifest and payload disagree; the checkpoint is corrupt"))
        if out is None:
            out = torch.empty(wanted.length, dtype=dtype or flat.dtype)
        lo = overlap.start - shard.offset
        out[filled:filled + overlap.length] = flat[lo:lo + overlap.length].to(out.dtype)
        filled += overlap.length
        cursor = overlap.end
    assert out is not None
    if filled != wanted.length:
        raise IncompleteCheckpointError(format_error("reshard.read_tensor_range", f"the shards of {record.key!r} cover only part of the range",
                                                     expected=wanted.length, observed=filled,
                                                     resolution="a payload file is absent or lost entries"))
    return out


def verify_files(directory: Path, manifest: CheckpointManifest, *, filenames: set[str] | None = None) -> dict[str, str]:
    """Check size and SHA-256 of every referenced file (or ``filenames``); returns the digests."""
    out = {}
    for name in sorted(filenames if filenames is not None else manifest.referenced_files()):
        _check_file(Path(directory), manifest, name, verify=True, where="reshard.verify_files")
        out[name] = manifest.files[name].sha256
    return out


def describe_reshard(manifest: CheckpointManifest, key: str, wanted: ShardRange) -> dict[str, Any]:
    """Which saved files/intervals would serve ``wanted`` of tensor ``key``."""
    record = manifest.tensors.get(key)
    if record is None:
        raise CheckpointError(format_error("reshard.describe_reshard", "unknown tensor key", expected=sorted(manifest.tensors)[:8],
                                           observed=key, resolution="compare the storage key with the manifest"))
    return {"key": key, "global_shape": list(record.global_shape), "wanted": [wanted.start, wanted.length],
            "sources": [{"file": s.file, "saved_rank": s.rank, "shard_range": [s.offset, s.length],
                         "overlap": [o.start, o.length]} for s, o in record.shards_overlapping(wanted)]}
