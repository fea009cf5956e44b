"""The checkpoint manifest: global tensors described as flat-interval shards.

Every saved tensor (model parameter, buffer or optimizer state) is one
``TensorRecord`` with its global shape and a list of ``ShardRecord`` intervals
``[offset, offset + length)`` of its flattened data, each stored under a key
in one ``rank-NNNNN.pt`` file.  Intervals are in *global* coordinates, which
is what lets a checkpoint written at one FSDP/DDP width be read at another.
Validation rejects overlaps, gaps, out-of-range shards and files without an
integrity record.  JSON layout (keys, nesting, ``sort_keys``, ``indent=2``)
matches ``src/hybrid_training/checkpoint/manifest.py:63-581``.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

from ..errors import CheckpointCorruptionError, CheckpointError, IncompleteCheckpointError, format_error
from ..utils.tensors import ShardRange, intersect_ranges
from .format import CURRENT_FORMAT_VERSION, validate_format_version, validate_shard_filename

__all__ = ["CheckpointManifest", "FileRecord", "ShardRecord", "TensorRecord"]


@dataclass(frozen=True)
class ShardRecord:
    rank: int
    file: str
    offset: int
    length: int
    key: str
    padding: int = 0

    def __post_init__(self) -> None:
        if self.offset < 0 or self.length < 0:
            raise CheckpointError(format_error("manifest.ShardRecord", "a shard record has a negative offset or length",
                                               expected="non-negative offset and length",
                                               observed=f"offset={self.offset}, length={self.length}", resolution="manifest.json has an unexpected structure"))
        validate_shard_filename(self.file)

    @property
    def range(self) -> ShardRange:
        return ShardRange(self.offset, self.length)

    def as_dict(self) -> dict[str, Any]:
        return {"rank": self.rank, "file": self.file, "offset": self.offset, "length": self.length, "key": self.key,
                "padding": self.padding}

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> ShardRecord:
        return cls(int(d["rank"]), str(d["file"]), int(d["offset"]), int(d["length"]), str(d["key"]), int(d.get("padding", 0)))


@dataclass
class TensorRecord:
    key: str
    name: str
    global_shape: tuple[int, ...]
    dtype: str
    category: str = "model"
    partition_dim: int | None = None
    tensor_parallel_size: int = 1
    tensor_parallel_rank: int = 0
    state_name: str = ""
    shards: list[ShardRecord] = field(default_factory=list)

    @property
    def numel(self) -> int:
        n = 1
        for d in self.global_shape:
            n *= d
        return n

    def covered_elements(self) -> int:
        """Size of the union of the shard intervals."""
        covered, end = 0, -1
        for lo, hi in sorted((s.offset, s.offset + s.length) for s in self.shards):
            if hi <= end:
                continue
            covered += hi - max(lo, end) if end > lo else hi - lo
            end = max(end, hi)
        return covered

    def validate(self) -> None:
        for s in self.shards:
            if s.offset + s.length > self.numel:
                raise CheckpointCorruptionError(format_error("manifest.TensorRecord.validate", f"a shard of {self.key!r} runs past the end",
                                                             expected=f"offset + length <= {self.numel}", observed=s.offset + s.length,
                                                             resolution="the numel in the manifest does not match the product of the shape"))
        total = sum(s.length for s in self.shards)
        covered = self.covered_elements()
        if total != covered:
            raise CheckpointCorruptionError(format_error("manifest.TensorRecord.validate",
                                                         f"the shards of {self.key!r} intersect: the same elements would be read from two places",
                                                         expected=f"{covered} elements, each in exactly one shard", observed=total,
                                                         resolution="a writer recorded an inconsistent layout; treat this checkpoint as unusable"))
        if covered != self.numel:
            raise IncompleteCheckpointError(format_error("manifest.TensorRecord.validate",
                                                         f"the shards of {self.key!r} leave elements of the tensor with no shard",
                                                         expected=f"{self.numel} elements", observed=covered,
                                                         resolution="the shards do not add up to the tensor, so it cannot be rebuilt"))

    def shards_overlapping(self, wanted: ShardRange) -> list[tuple[ShardRecord, ShardRange]]:
        out = []
        for s in sorted(self.shards, key=lambda s: s.offset):
            o = intersect_ranges(s.range, wanted)
            if o is not None:
                out.append((s, o))
        return out

    def as_dict(self) -> dict[str, Any]:
        return {"key": self.key, "name": self.name, "global_shape": list(self.global_shape), "numel": self.numel, "dtype": self.dtype,
                "category": self.category, "partition_dim": self.partition_dim, "tensor_parallel_size": self.tensor_parallel_size,
                "tensor_parallel_rank": self.tensor_parallel_rank, "state_name": self.state_name,
                "shards": [s.as_dict() for s in sorted(self.shards, key=lambda s: s.offset)]}

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> TensorRecord:
        pdim = d.get("partition_dim")
        return cls(str(d["key"]), str(d["name"]), tuple(int(x) for x in d["global_shape"]), str(d["dtype"]),
                   str(d.get("category", "model")), None if pdim is None else int(pdim), int(d.get("tensor_parallel_size", 1)),
                   int(d.get("tensor_parallel_rank", 0)), str(d.get("state_name", "")),
                   [ShardRecord.from_dict(s) for s in d.get("shards", [])])


@dataclass(frozen=True)
class FileRecord:
    name: str
    sha256: str
    bytes: int

    def as_dict(self) -> dict[str, Any]:
        return {"name": self.name, "sha256": self.sha256, "bytes": self.bytes}

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> FileRecord:
        return cls(validate_shard_filename(str(d["name"])), str(d["sha256"]), int(d["bytes"]))


@dataclass
class CheckpointManifest:
    format_version: str = CURRENT_FORMAT_VERSION
    writer_world_size: int = 1
    topology: dict[str, Any] = field(default_factory=dict)
    step: int = 0
    tensors: dict[str, TensorRecord] = field(default_factory=dict)
    files: dict[str, FileRecord] = field(default_factory=dict)
    complete: bool = False
    created_by: str = ""

    def add_shard(self, record: TensorRecord, shard: ShardRecord) -> None:
        existing = self.tensors.get(record.key)
        if existing is None:
            self.tensors[record.key] = TensorRecord(record.key, record.name, record.global_shape, record.dtype, record.category,
                                                    record.partition_dim, record.tensor_parallel_size, record.tensor_parallel_rank,
                                                    record.state_name, [shard])
            return
        if existing.global_shape != record.global_shape or existing.dtype != record.dtype:
            raise CheckpointCorruptionError(format_error(
                "manifest.add_shard", f"the records of two ranks disagree about tensor {record.key!r} differently",
                expected=f"shape={existing.global_shape}, dtype={existing.dtype}",
                observed=f"shape={record.global_shape}, dtype={record.dtype}",
                resolution="every rank must build the model from the same configuration"))
        existing.shards.append(shard)

    def validate(self) -> None:
        validate_format_version(self.format_version)
        if not self.complete:
            raise IncompleteCheckpointError(format_error("manifest.validate", "the manifest is not marked complete; the writer did not finish",
                                                         expected=True, observed=self.complete,
                                                         resolution="use an older checkpoint"))
        for record in self.tensors.values():
            record.validate()
            for s in record.shards:
                if s.file not in self.files:
                    raise IncompleteCheckpointError(format_error("manifest.validate",
                                                                 f"tensor {record.key!r} references file {s.file!r} without an integrity record",
                                                                 expected=sorted(self.files), observed=s.file,
                                                                 resolution="manifest.json is incomplete or was edited"))

    def referenced_files(self) -> set[str]:
        return {s.file for r in self.tensors.values() for s in r.shards}

    def tensors_by_category(self, category: str) -> dict[str, TensorRecord]:
        return {k: v for k, v in self.tensors.items() if v.category == category}

    def as_dict(self) -> dict[str, Any]:
        return {"format_version": self.format_version, "created_by": self.created_by, "writer_world_size": self.writer_world_size,
                "topology": self.topology, "step": self.step, "complete": self.complete,
                "tensors": {k: self.tensors[k].as_dict() for k in sorted(self.tensors)},
                "files": {k: self.files[k].as_dict() for k in sorted(self.files)}}

    def to_json(self, *, indent: int = 2) -> str:
        return json.dumps(self.as_dict(), indent=indent, sort_keys=True)

    def write(self, path: Path) -> Path:
        path.write_text(self.to_json(), encoding="utf-8")
        return path

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> CheckpointManifest:
        try:
            return cls(str(d["format_version"]), int(d.get("writer_world_size", 1)), dict(d.get("topology", {})), int(d.get("step", 0)),
                       {k: TensorRecord.from_dict(v) for k, v in d.get("tensors", {}).items()},
                       {k: FileRecord.from_dict(v) for k, v in d.get("files", {}).items()}, bool(d.get("complete", False)),
                       str(d.get("created_by", "")))
        except (KeyError, TypeError, ValueError) as exc:
            raise CheckpointError(format_error("manifest.from_dict", "manifest.json has an unexpected structure", expected="a manifest written by this format",
                                               observed=repr(exc), resolution="manifest.json lacks fields that every manifest has")) from exc

    @classmethod
    def read(cls, path: Path) -> CheckpointManifest:
        if not path.is_file():
            raise IncompleteCheckpointError(format_error("manifest.read", "no manifest found; it is written last, so the checkpoint "
                                                         "was never completed", expected=str(path), observed="missing",
                                                         resolution="use an older checkpoint"))
        try:
            payload = json.loads(path.read_text(encoding="utf-8"))
        except json.JSONDecodeError as exc:
            raise CheckpointError(format_error("manifest.read", "manifest.json cannot be parsed as JSON", expected="a JSON object",
                                               observed=str(exc), resolution="the file is corrupt")) from exc
        if not isinstance(payload, dict):
            raise CheckpointError(format_error("manifest.read", "manifest.json does not hold a JSON object at the top level", expected="object",
                                               observed=type(payload).__name__, resolution="the file is corrupt"))
        return cls.from_dict(payload)

    def summary(self) -> str:
        by = {c: len(self.tensors_by_category(c)) for c in ("model", "optimizer", "buffer")}
        rows = [("saved at step", self.step), ("ranks that wrote it", self.writer_world_size), ("grid", self.topology),
                ("finished", self.complete), ("model tensors", by["model"]), ("optimizer tensors", by["optimizer"]),
                ("buffers", by["buffer"]), ("elements in all", sum(r.numel for r in self.tensors.values())),
                ("rank files", len(self.files))]
        lines = [f"format v{self.format_version}, by {self.created_by or 'unknown'}"] + [f"  {k:<20} {v}" for k, v in rows]
        return "\n".join(lines)
