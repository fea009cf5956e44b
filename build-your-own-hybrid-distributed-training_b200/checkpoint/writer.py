"""Collective checkpoint writing: staged, checksummed, manifest-last, atomically renamed.

The protocol (``src/hybrid_training/checkpoint/writer.py:147-695``) makes every
rank raise together or none at all:

1. rank 0 decides (new directory? staging token) and all ranks adopt its
   verdict; an existing destination is an error everywhere;
2. rank 0 creates ``.staging-<name>-<token>``; the outcome is shared; barrier;
3. each rank writes ``rank-NNNNN.pt`` holding its pieces, keyed
   ``"<category>::<key>@<offset>"`` (model / buffer / optimizer), plus its RNG
   state under ``"rng::<name>"``; model and optimizer pieces come only from
   ranks with ``data_parallel == 0`` and ``sequence == 0`` (their replicas hold
   identical data); per-file SHA-256 and size are exchanged;
4. rank 0 builds and validates the manifest, writes ``metadata.json`` then
   ``manifest.json`` (last), and renames the staging directory into place;
   the outcome is shared; barrier; optional pruning; barrier.
"""

from __future__ import annotations

import json
import shutil
import time
import uuid
from dataclasses import asdict
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
    file_digest,
    shard_filename,
    staging_directory_name,
    step_from_directory_name,
)
from .manifest import CheckpointManifest, FileRecord, ShardRecord, TensorRecord

__all__ = ["CheckpointWriteResult", "find_latest_checkpoint", "prune_checkpoints", "save_checkpoint"]

_LOG = get_logger(__name__)
_RNG = "rng::"


class CheckpointWriteResult:
    def __init__(self, path: Path, step: int, seconds: float, bytes_written: int, num_tensors: int) -> None:
        self.path, self.step, self.seconds, self.bytes_written, self.num_tensors = path, step, seconds, bytes_written, num_tensors

    def __repr__(self) -> str:
        return (f"CheckpointWriteResult(path={self.path.name!r}, step={self.step}, {self.seconds:.3f}s, {self.bytes_written} bytes, "
                f"{self.num_tensors} tensors)")


def _writes_replicated_tensors(context: DistributedContext) -> bool:
    c = context.topology.coordinates_of(context.rank)
    return c.data_parallel == 0 and c.sequence == 0


def _agree(value: Any, context: DistributedContext) -> Any:
    """Everyone adopts rank 0's value."""
    return all_gather_object_in_group(value, context.group("world"))[0]


def save_checkpoint(directory: str | Path, *, model: HybridModel, context: DistributedContext, state: TrainingState,
                    optimizer: ShardedOptimizer | None = None, config: ExperimentConfig | None = None,
                    scheduler_state: dict[str, Any] | None = None, scaler_state: dict[str, Any] | None = None,
                    extra_metadata: dict[str, Any] | None = None, save_optimizer: bool = True, save_rng: bool = True,
                    keep_last: int = 0) -> CheckpointWriteResult:
    start = time.perf_counter()
    root = Path(directory)
    final_name = checkpoint_directory_name(state.step)
    final = root / final_name
    verdict = _agree({"token": uuid.uuid4().hex[:12], "exists": final.exists()} if context.is_primary else None, context)
    if verdict["exists"]:
        raise CheckpointError(format_error("checkpoint.save", "the destination checkpoint already exists", rank=context.rank,
                                           world_size=context.world_size, expected="a fresh directory", observed=str(final),
                                           resolution="remove the existing checkpoint or save at a different step"))
    staging = root / staging_directory_name(final_name, verdict["token"])
    error = ""
    if context.is_primary:
        try:
            staging.mkdir(parents=True, exist_ok=True)
        except OSError as exc:
            error = str(exc)
    error = _agree(error, context)
    if error:
        raise CheckpointError(format_error("checkpoint.save", "the staging directory could not be created", rank=context.rank,
                                           world_size=context.world_size, expected=str(staging), observed=error,
                                           resolution="check permissions and free space on the checkpoint filesystem"))
    context.barrier("world", label="checkpoint-staging-created")
    payload, records, scalars = _collect_payload(model=model, optimizer=optimizer, context=context, save_optimizer=save_optimizer,
                                                 save_rng=save_rng)
    name = shard_filename(context.rank)
    path = staging / name
    torch.save(payload, path)
    size = path.stat().st_size
    mine = {"file": {"name": name, "sha256": file_digest(path), "bytes": size}, "records": records, "optimizer_scalars": scalars}
    gathered = all_gather_object_in_group(mine, context.group("world"))
    context.barrier("world", label="checkpoint-payloads-written")
    error = ""
    if context.is_primary:
        try:
            _publish(context=context, state=state, config=config, scheduler_state=scheduler_state, scaler_state=scaler_state,
                     extra_metadata=extra_metadata, gathered=gathered, save_rng=save_rng, staging=staging, final=final)
        except Exception as exc:
            error = f"{type(exc).__name__}: {exc}"
    error = _agree(error, context)
    if error:
        raise CheckpointError(format_error("checkpoint.save", "the checkpoint could not be published; nothing was renamed into place",
                                           rank=context.rank, world_size=context.world_size,
                                           expected="a validated manifest covering every tensor exactly once", observed=error,
                                           resolution=f"read rank 0's error; staging directory {staging.name!r} is kept for inspection"))
    context.barrier("world", label="checkpoint-published")
    if context.is_primary and keep_last > 0:
        prune_checkpoints(root, keep_last=keep_last)
    context.barrier("world", label="checkpoint-pruned")
    return CheckpointWriteResult(final, state.step, time.perf_counter() - start, size, len(records))


def _publish(*, context: DistributedContext, state: TrainingState, config: ExperimentConfig | None,
             scheduler_state: dict[str, Any] | None, scaler_state: dict[str, Any] | None, extra_metadata: dict[str, Any] | None,
             gathered: list[dict[str, Any]], save_rng: bool, staging: Path, final: Path) -> None:
    manifest = CheckpointManifest(CURRENT_FORMAT_VERSION, context.world_size, context.topology.summary(), state.step,
                                  created_by=f"hybrid_training {__version__}")
    for entry in gathered:
        fr = FileRecord.from_dict(entry["file"])
        manifest.files[fr.name] = fr
        for item in entry["records"]:
            manifest.add_shard(
                TensorRecord(item["key"], item["name"], tuple(item["global_shape"]), item["dtype"], item["category"],
                             item["partition_dim"], item["tensor_parallel_size"], item["tensor_parallel_rank"], item["state_name"]),
                ShardRecord(item["rank"], item["file"], item["offset"], item["length"], item["storage_key"], item.get("padding", 0)))
    manifest.complete = True
    manifest.validate()
    for name in manifest.referenced_files():
        if not (staging / name).is_file():
            raise CheckpointError(format_error("checkpoint.save", "a rank reported a file that is not in the staging directory",
                                               rank=context.rank, world_size=context.world_size, expected=name, observed="missing",
                                               resolution="check for a filesystem error on the reporting rank"))
    metadata = _build_metadata(context=context, state=state, config=config, scheduler_state=scheduler_state,
                               scaler_state=scaler_state, extra_metadata=extra_metadata, gathered=gathered, save_rng=save_rng)
    (staging / METADATA_FILENAME).write_text(_dump_json(metadata), encoding="utf-8")
    manifest.write(staging / MANIFEST_FILENAME)
    staging.replace(final)
    _LOG.info("checkpoint written: %s (%d tensors, %d files)", final, len(manifest.tensors), len(manifest.files))


def _collect_payload(*, model: HybridModel, optimizer: ShardedOptimizer | None, context: DistributedContext, save_optimizer: bool,
                     save_rng: bool) -> tuple[dict[str, torch.Tensor], list[dict[str, Any]], dict[str, Any]]:
    fname = shard_filename(context.rank)
    info_of = model.parameter_parallel_info()
    payload: dict[str, torch.Tensor] = {}
    records: list[dict[str, Any]] = []
    scalars: dict[str, Any] = {}

    def add(key: str, name: str, shape: tuple[int, ...], offset: int, data: torch.Tensor, category: str, state_name: str = "") -> None:
        info = info_of.get(name)
        storage_key = f"{category}::{key}@{offset}"
        payload[storage_key] = data.detach().cpu().reshape(-1).clone()
        records.append({"key": key, "name": name, "global_shape": list(shape), "dtype": str(data.dtype), "category": category,
                        "partition_dim": None if info is None else info.partition_dim,
                        "tensor_parallel_size": 1 if info is None else info.tensor_parallel_size,
                        "tensor_parallel_rank": 0 if info is None else info.tensor_parallel_rank, "state_name": state_name,
                        "rank": context.rank, "file": fname, "offset": offset, "length": int(data.numel()), "storage_key": storage_key})

    if _writes_replicated_tensors(context):
        for name, piece in model.sharded_state_dict().items():
            info = info_of.get(name)
            add(info.storage_key if info else name, name, piece.global_shape, piece.offset, piece.data, "model")
        for name, buf in model.buffers_state_dict().items():
            add(name, name, tuple(buf.shape), 0, buf.reshape(-1), "buffer")
        if save_optimizer and optimizer is not None:
            layouts = model.optimizer_parameter_layout()
            inner_state = optimizer.inner.state
            for index, param in enumerate(optimizer.parameters):
                entry = inner_state.get(param)
                if not entry:
                    continue
                for state_name, value in entry.items():
                    if not torch.is_tensor(value) or value.numel() != param.numel():
                        scalar = _as_scalar(value)
                        if state_name in scalars and scalars[state_name] != scalar:
                            raise CheckpointError(format_error(
                                "checkpoint.save", f"optimizer state {state_name!r} differs between parameters; the format stores "
                                "one value per state name", rank=context.rank, expected=scalars[state_name], observed=scalar,
                                resolution="step every parameter together"))
                        scalars[state_name] = scalar
                        continue
                    flat = value.detach().reshape(-1)
                    for item in layouts[index]:
                        info = info_of.get(item.name)
                        base = info.storage_key if info else item.name
                        add(f"{base}::{state_name}", item.name, item.global_shape, item.parameter_offset,
                            flat[item.local_offset:item.local_offset + item.length], "optimizer", state_name)
    if save_rng:
        for name, t in rng_state_to_serialisable(capture_rng_state())["tensors"].items():
            payload[f"{_RNG}{name}"] = t
    return payload, records, scalars


def _as_scalar(value: Any) -> Any:
    if torch.is_tensor(value):
        return value.item() if value.numel() == 1 else [float(v) for v in value.reshape(-1).tolist()]
    return value


def _build_metadata(*, context: DistributedContext, state: TrainingState, config: ExperimentConfig | None,
                    scheduler_state: dict[str, Any] | None, scaler_state: dict[str, Any] | None, extra_metadata: dict[str, Any] | None,
                    gathered: list[dict[str, Any]], save_rng: bool) -> dict[str, Any]:
    scalars: dict[str, Any] = {}
    for entry in gathered:
        scalars.update(entry.get("optimizer_scalars", {}))
    return {"format_version": CURRENT_FORMAT_VERSION, "created_by": f"hybrid_training {__version__}",
            "training_state": state.as_dict(), "scheduler": scheduler_state or {}, "scaler": scaler_state or {},
            "config": None if config is None else config.to_dict(), "topology": context.topology.summary(),
            "world_size": context.world_size, "backend": context.backend,
            "rng": {"saved": save_rng, "ranks": list(range(context.world_size)) if save_rng else [],
                    "meta": rng_state_to_serialisable(capture_rng_state())["meta"] if save_rng else {}},
            "optimizer_scalars": scalars, "extra": extra_metadata or {}}


def _dump_json(payload: dict[str, Any]) -> str:
    def default(v: Any) -> Any:
        if isinstance(v, (set, frozenset, tuple)):
            return list(v)
        if hasattr(v, "as_dict"):
            return v.as_dict()
        if hasattr(v, "__dataclass_fields__"):
            return asdict(v)
        raise TypeError(f"checkpoint metadata must be JSON-serialisable; {type(v).__name__} is not (tensors belong in payload files)")

    return json.dumps(payload, indent=2, sort_keys=True, default=default, allow_nan=False)


def prune_checkpoints(root: str | Path, *, keep_last: int) -> list[Path]:
    """Delete all but the newest ``keep_last`` complete-looking checkpoint directories."""
    base = Path(root)
    if keep_last <= 0 or not base.is_dir():
        return []
    found = sorted((s, c) for c in base.iterdir() if c.is_dir() and (s := step_from_directory_name(c.name)) is not None)
    removed = []
    for _, path in found[:max(len(found) - keep_last, 0)]:
        shutil.rmtree(path, ignore_errors=True)
        removed.append(path)
        _LOG.info("pruned old checkpoint %s", path.name)
    return removed


def find_latest_checkpoint(root: str | Path) -> Path | None:
    """Newest ``checkpoint-step-*`` directory that has a manifest (i.e. was published)."""
    base = Path(root)
    if not base.is_dir():
        return None
    best: tuple[int, Path] | None = None
    for child in sorted(base.iterdir()):
        if not child.is_dir() or not CHECKPOINT_DIRECTORY_PATTERN.match(child.name) or not (child / MANIFEST_FILENAME).is_file():
            continue
        step = step_from_directory_name(child.name)
        if step is not None and (best is None or step > best[0]):
            best = (step, child)
    return None if best is None else best[1]
