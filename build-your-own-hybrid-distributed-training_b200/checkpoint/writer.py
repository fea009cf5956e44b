"""Collective checkpoint writer.

The on-disk result is the reference's format (``src/hybrid_training/checkpoint/writer.py:147-695``
writes the same directory): ``checkpoint-step-NNNNNN/`` with one ``rank-NNNNN.pt`` payload per
rank, ``metadata.json`` and ``manifest.json``, built in a ``.staging-<final>-<token>`` directory
that is renamed into place only after the manifest, written last, has validated.  The code here is
organised differently:

* A save is a :class:`_SaveTransaction` that every rank runs in lock-step through four phases
  (reserve, write, commit, retire).  Each phase ends in a *vote*: every rank contributes
  ``(ok, reason)`` in one object all-gather and every rank evaluates the same list, so a failure on
  any rank -- not only on the coordinator -- makes all ranks raise the same error before the next
  phase starts.  The coordinator (global rank 0) is the only rank that touches shared directory
  state (create the staging directory, write the manifest, rename, prune).
* Payload bytes are hashed while they stream to disk (:class:`_DigestingFile`), then the file is
  fsync'ed; nothing re-reads a payload to checksum it.
* :class:`_PayloadBuilder` turns the model's global-coordinate pieces, its buffers, the optimizer
  state (one flat interval per parameter piece, keyed ``"<storage key>::<state>"``) and this rank's
  RNG streams into the payload dictionary plus one manifest record per piece.  Replicated tensors
  are written by the ranks at ``data_parallel == 0`` and ``sequence == 0`` only; RNG state by every
  rank.
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil
import time
import uuid
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any

import torch

from .. import __version__
from ..config import ExperimentConfig
from ..distributed.collectives import all_gather_object_in_group
from ..distributed.context import DistributedContext
from ..errors import CheckpointError, format_error
from ..logging import get_logger
from ..optim.sharded_optimizer import ShardedOptimizer
from ..parallel.hybrid import HybridModel
from ..training.state import TrainingState
from ..utils.reproducibility import capture_rng_state, rng_state_to_serialisable
from .format import (
    CHECKPOINT_DIRECTORY_PATTERN,
    CURRENT_FORMAT_VERSION,
    MANIFEST_FILENAME,
    METADATA_FILENAME,
    checkpoint_directory_name,
    shard_filename,
    staging_directory_name,
    step_from_directory_name,
)
from .manifest import CheckpointManifest, FileRecord, ShardRecord, TensorRecord

__all__ = ["CheckpointWriteResult", "find_latest_checkpoint", "prune_checkpoints", "save_checkpoint"]

_LOG = get_logger(__name__)
_RNG_PREFIX = "rng::"
_COORDINATOR = 0


@dataclass(frozen=True)
class CheckpointWriteResult:
    """What one rank's part of a save produced."""

    path: Path
    step: int
    seconds: float
    bytes_written: int
    num_tensors: int
    sha256: str = ""

    def __repr__(self) -> str:
        return (f"CheckpointWriteResult({self.path.name}, step {self.step}: {self.num_tensors} pieces, "
                f"{self.bytes_written} bytes in {self.seconds:.3f}s)")


class _DigestingFile:
    """Binary file that feeds every written byte to SHA-256 and counts it."""

    def __init__(self, path: Path) -> None:
        self._file = path.open("wb")
        self._hash = hashlib.sha256()
        self.size = 0

    def write(self, data: Any) -> int:
        view = memoryview(data)
        self._hash.update(view)
        self.size += view.nbytes
        return self._file.write(view)

    def flush(self) -> None:
        self._file.flush()

    def finish(self) -> str:
        """Flush to stable storage, close, and return the hex digest."""
        self._file.flush()
        os.fsync(self._file.fileno())
        self._file.close()
        return self._hash.hexdigest()

    def abandon(self) -> None:
        if not self._file.closed:
            self._file.close()


@dataclass
class _PayloadBuilder:
    """Collects this rank's tensors (payload) and the manifest records that describe them."""

    rank: int
    file_name: str
    parallel_info: dict[str, Any]
    tensors: dict[str, torch.Tensor] = field(default_factory=dict)
    records: list[dict[str, Any]] = field(default_factory=list)
    scalars: dict[str, Any] = field(default_factory=dict)

    def piece(self, *, category: str, key: str, name: str, global_shape: tuple[int, ...], offset: int, values: torch.Tensor,
              state_name: str = "") -> None:
        storage_key = f"{category}::{key}@{offset}"
        flat = values.detach().reshape(-1).to("cpu", copy=True)
        self.tensors[storage_key] = flat
        info = self.parallel_info.get(name)
        self.records.append({
            "key": key, "name": name, "global_shape": [int(s) for s in global_shape], "dtype": str(flat.dtype),
            "category": category, "state_name": state_name,
            "partition_dim": info.partition_dim if info is not None else None,
            "tensor_parallel_size": info.tensor_parallel_size if info is not None else 1,
            "tensor_parallel_rank": info.tensor_parallel_rank if info is not None else 0,
            "rank": self.rank, "file": self.file_name, "offset": int(offset), "length": int(flat.numel()),
            "storage_key": storage_key})

    def storage_key_of(self, name: str) -> str:
        info = self.parallel_info.get(name)
        return info.storage_key if info is not None else name

    def add_model(self, model: HybridModel) -> None:
        for name, piece in model.sharded_state_dict().items():
            self.piece(category="model", key=self.storage_key_of(name), name=name, global_shape=piece.global_shape,
                       offset=piece.offset, values=piece.data)
        for name, buf in model.buffers_state_dict().items():
            self.piece(category="buffer", key=name, name=name, global_shape=tuple(buf.shape), offset=0, values=buf)

    def add_optimizer(self, model: HybridModel, optimizer: ShardedOptimizer) -> None:
        layouts = model.optimizer_parameter_layout()
        for index, param in enumerate(optimizer.parameters):
            for state_name, value in (optimizer.inner.state.get(param) or {}).items():
                if torch.is_tensor(value) and value.numel() == param.numel():
                    flat = value.detach().reshape(-1)
                    for item in layouts[index]:
                        self.piece(category="optimizer", key=f"{self.storage_key_of(item.name)}::{state_name}", name=item.name,
                                   global_shape=item.global_shape, offset=item.parameter_offset,
                                   values=flat[item.local_offset:item.local_offset + item.length], state_name=state_name)
                else:
                    self._scalar(state_name, value)

    def _scalar(self, state_name: str, value: Any) -> None:
        if torch.is_tensor(value):
            value = value.item() if value.numel() == 1 else [float(v) for v in value.reshape(-1).tolist()]
        previous = self.scalars.setdefault(state_name, value)
        if previous != value:
            raise CheckpointError(format_error(
                "checkpoint.save", f"the per-parameter optimizer scalar {state_name!r} is not the same for every parameter, but "
                "the checkpoint keeps a single value per scalar name", rank=self.rank, expected=previous, observed=value,
                resolution="save only after optimizer steps that updated every parameter (e.g. not mid-way through a "
                           "partial step)"))

    def add_rng(self) -> None:
        for name, t in rng_state_to_serialisable(capture_rng_state())["tensors"].items():
            self.tensors[_RNG_PREFIX + name] = t


class _SaveTransaction:
    """One save, driven through reserve -> write -> commit -> retire on every rank."""

    def __init__(self, root: Path, context: DistributedContext, step: int) -> None:
        self.root = root
        self.context = context
        self.step = step
        self.final = root / checkpoint_directory_name(step)
        self.staging: Path | None = None
        self.started = time.perf_counter()

    # -- voting --------------------------------------------------------------------------------------------------
    def _vote(self, phase: str, problem: str | None, payload: Any = None) -> list[dict[str, Any]]:
        """Every rank shares ``problem`` (None = fine); all raise together when any rank reported one."""
        ballots = all_gather_object_in_group({"rank": self.context.rank, "problem": problem, "payload": payload},
                                             self.context.group("world"))
        failed = [b for b in ballots if b["problem"]]
        if failed:
            first = failed[0]
            raise CheckpointError(format_error(
                f"checkpoint.save[{phase}]", f"{len(failed)} rank(s) could not complete the {phase} phase; the checkpoint "
                "was not published", rank=self.context.rank, world_size=self.context.world_size,
                expected=f"every rank to finish {phase}", observed=f"rank {first['rank']}: {first['problem']}",
                resolution=_PHASE_HINTS[phase]))
        return ballots

    # -- phases ----------------------------------------------------------------------------------------------------
    def reserve(self) -> None:
        problem, token = None, None
        if self.context.rank == _COORDINATOR:
            token = uuid.uuid4().hex[:12]
            if self.final.exists():
                problem = f"{self.final} is already present"
            else:
                try:
                    (self.root / staging_directory_name(self.final.name, token)).mkdir(parents=True)
                except OSError as exc:
                    problem = f"creating the staging directory failed ({exc})"
        ballots = self._vote("reserve", problem, token)
        self.staging = self.root / staging_directory_name(self.final.name, ballots[_COORDINATOR]["payload"])

    def write(self, builder: _PayloadBuilder) -> tuple[dict[str, Any], list[dict[str, Any]]]:
        assert self.staging is not None
        problem, mine = None, None
        target = self.staging / builder.file_name
        sink = None
        try:
            sink = _DigestingFile(target)
            torch.save(builder.tensors, sink)
            digest = sink.finish()
            mine = {"file": {"name": builder.file_name, "sha256": digest, "bytes": sink.size}, "records": builder.records,
                    "optimizer_scalars": builder.scalars}
        except Exception as exc:  # reported through the vote so that every rank raises
            if sink is not None:
                sink.abandon()
            problem = f"writing {target.name} failed ({type(exc).__name__}: {exc})"
        ballots = self._vote("write", problem, mine)
        return mine, [b["payload"] for b in ballots]

    def commit(self, metadata: dict[str, Any], contributions: list[dict[str, Any]]) -> None:
        problem = None
        if self.context.rank == _COORDINATOR:
            try:
                _publish(self.staging, self.final, self.context, self.step, metadata, contributions)
            except Exception as exc:
                problem = f"{type(exc).__name__}: {exc} (staging directory {self.staging.name} left for inspection)"
        self._vote("commit", problem)

    def retire(self, keep_last: int) -> None:
        problem = None
        if self.context.rank == _COORDINATOR and keep_last > 0:
            try:
                prune_checkpoints(self.root, keep_last=keep_last)
            except OSError as exc:
                problem = f"pruning failed ({exc})"
        self._vote("retire", problem)


_PHASE_HINTS = {
    "reserve": "pick another step or delete the old directory, and make sure the checkpoint root is writable",
    "write": "look at the failing rank's filesystem: free space, quota and permissions of the checkpoint root",
    "commit": "the coordinator's manifest or rename failed; its message names the cause",
    "retire": "the new checkpoint is published; remove old checkpoint directories by hand",
}


def _publish(staging: Path, final: Path, context: DistributedContext, step: int, metadata: dict[str, Any],
             contributions: list[dict[str, Any]]) -> None:
    """Coordinator only: manifest from every rank's records, metadata, manifest last, then rename."""
    manifest = CheckpointManifest(CURRENT_FORMAT_VERSION, context.world_size, context.topology.summary(), step,
                                  created_by=f"hybrid_training {__version__}")
    for part in contributions:
        record = FileRecord.from_dict(part["file"])
        on_disk = staging / record.name
        if not on_disk.is_file() or on_disk.stat().st_size != record.bytes:
            raise CheckpointError(format_error("checkpoint.save[commit]", "a payload file is missing or has a different size "
                                               "than its writer reported", rank=context.rank, expected=f"{record.name}: "
                                               f"{record.bytes} bytes", observed="missing" if not on_disk.is_file()
                                               else f"{on_disk.stat().st_size} bytes",
                                               resolution="the staging directory is not shared by all ranks, or a disk "
                                                          "error occurred; use a filesystem that every rank sees"))
        manifest.files[record.name] = record
        for r in part["records"]:
            tensor = TensorRecord(r["key"], r["name"], tuple(r["global_shape"]), r["dtype"], r["category"], r["partition_dim"],
                                  r["tensor_parallel_size"], r["tensor_parallel_rank"], r["state_name"])
            manifest.add_shard(tensor, ShardRecord(r["rank"], r["file"], r["offset"], r["length"], r["storage_key"],
                                                   r.get("padding", 0)))
    manifest.complete = True
    manifest.validate()
    (staging / METADATA_FILENAME).write_text(_to_json(metadata), encoding="utf-8")
    manifest.write(staging / MANIFEST_FILENAME)  # written last: its presence marks a finished directory
    os.replace(staging, final)
    _LOG.info("published %s: %d tensors in %d payload files", final, len(manifest.tensors), len(manifest.files))


def _metadata(*, context: DistributedContext, state: TrainingState, config: ExperimentConfig | None,
              scheduler_state: dict[str, Any] | None, scaler_state: dict[str, Any] | None, extra: dict[str, Any] | None,
              contributions: list[dict[str, Any]], save_rng: bool) -> dict[str, Any]:
    scalars: dict[str, Any] = {}
    for part in contributions:
        scalars.update(part.get("optimizer_scalars") or {})
    rng = {"saved": False, "ranks": [], "meta": {}}
    if save_rng:
        rng = {"saved": True, "ranks": list(range(context.world_size)),
               "meta": rng_state_to_serialisable(capture_rng_state())["meta"]}
    return {"format_version": CURRENT_FORMAT_VERSION, "created_by": f"hybrid_training {__version__}",
            "training_state": state.as_dict(), "scheduler": dict(scheduler_state or {}), "scaler": dict(scaler_state or {}),
            "config": config.to_dict() if config is not None else None, "topology": context.topology.summary(),
            "world_size": context.world_size, "backend": context.backend, "rng": rng, "optimizer_scalars": scalars,
            "extra": dict(extra or {})}


def _to_json(obj: dict[str, Any]) -> str:
    def encode(value: Any) -> Any:
        if isinstance(value, (tuple, set, frozenset)):
            return list(value)
        if hasattr(value, "as_dict"):
            return value.as_dict()
        if hasattr(value, "__dataclass_fields__"):
            return asdict(value)
        raise TypeError(f"{type(value).__name__} cannot go into metadata.json; tensors are stored in the payload files")

    return json.dumps(obj, indent=2, sort_keys=True, default=encode, allow_nan=False)


def save_checkpoint(directory: str | Path, *, model: HybridModel, context: DistributedContext, state: TrainingState,
                    optimizer: ShardedOptimizer | None = None, config: ExperimentConfig | None = None,
                    scheduler_state: dict[str, Any] | None = None, scaler_state: dict[str, Any] | None = None,
                    extra_metadata: dict[str, Any] | None = None, save_optimizer: bool = True, save_rng: bool = True,
                    keep_last: int = 0) -> CheckpointWriteResult:
    """Write ``checkpoint-step-<step>`` under ``directory``; collective over the world group.

    Every rank returns normally or every rank raises :class:`CheckpointError`; a failed save
    leaves no directory named like a checkpoint (a staging directory may remain for inspection).
    """
    tx = _SaveTransaction(Path(directory), context, state.step)
    tx.reserve()
    builder = _PayloadBuilder(context.rank, shard_filename(context.rank), model.parameter_parallel_info())
    coords = context.topology.coordinates_of(context.rank)
    if coords.data_parallel == 0 and coords.sequence == 0:  # replicas along dp / seq hold identical tensors
        builder.add_model(model)
        if save_optimizer and optimizer is not None:
            builder.add_optimizer(model, optimizer)
    if save_rng:
        builder.add_rng()
    mine, contributions = tx.write(builder)
    metadata = _metadata(context=context, state=state, config=config, scheduler_state=scheduler_state,
                         scaler_state=scaler_state, extra=extra_metadata, contributions=contributions, save_rng=save_rng)
    tx.commit(metadata, contributions)
    tx.retire(keep_last)
    return CheckpointWriteResult(tx.final, state.step, time.perf_counter() - tx.started, int(mine["file"]["bytes"]),
                                 len(builder.records), mine["file"]["sha256"])


def prune_checkpoints(root: str | Path, *, keep_last: int) -> list[Path]:
    """Remove checkpoint directories older than the newest ``keep_last``; returns what was removed."""
    base = Path(root)
    if keep_last <= 0 or not base.is_dir():
        return []
    by_step = {}
    for child in base.iterdir():
        step = step_from_directory_name(child.name) if child.is_dir() else None
        if step is not None:
            by_step[step] = child
    doomed = [by_step[s] for s in sorted(by_step)[:-keep_last]] if len(by_step) > keep_last else []
    for path in doomed:
        shutil.rmtree(path, ignore_errors=True)
        _LOG.info("removed checkpoint %s (keep_last=%d)", path.name, keep_last)
    return doomed


def find_latest_checkpoint(root: str | Path) -> Path | None:
    """The published checkpoint (one with a manifest) with the highest step under ``root``, if any."""
    base = Path(root)
    if not base.is_dir():
        return None
    published = [(step_from_directory_name(c.name), c) for c in base.iterdir()
                 if c.is_dir() and CHECKPOINT_DIRECTORY_PATTERN.match(c.name) and (c / MANIFEST_FILENAME).is_file()]
    return max(published, key=lambda sc: sc[0])[1] if published else None
