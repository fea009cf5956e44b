"""Explicit-group collective wrappers with communication accounting.

Contract (same as ``src/hybrid_training/distributed/collectives.py:1-954``):

* every wrapper takes a :class:`GroupHandle`; there is no default group;
* single-member groups short-circuit (no communicator exists for them);
* ``AVG`` means *pre-divide by the group size, then sum*.  On NCCL the divide is
  folded into the reduction with a pre-multiplied sum, on Gloo it is a
  separate ``div_`` (Gloo has no AVG);
* inputs must be contiguous;
* :class:`CommunicationRecorder` counts calls, bytes, launch time and wait time
  per ``"op/group"``; waiting never increments ``calls``.
"""

from __future__ import annotations

import time
from collections.abc import Callable, Iterable, Iterator, Sequence
from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Any

import torch
import torch.distributed as dist

from ..errors import CollectiveError, ParameterConsistencyError, format_error
from ..logging import get_logger
from .groups import GroupHandle, validate_group_membership

__all__ = [
    "observe_collectives",
    "record_collective",
    "AsyncWork",
    "CommunicationRecorder",
    "CommunicationStats",
    "ReduceOp",
    "all_gather_object_in_group",
    "all_gather_tensor",
    "all_reduce",
    "all_to_all_tensor",
    "assert_metadata_consistent",
    "assert_tensor_consistent",
    "broadcast",
    "concat_shard_sizes",
    "recv_tensor",
    "reduce_scatter_tensor",
    "send_tensor",
    "sum_scalar",
    "wait_all",
]

_LOG = get_logger(__name__)


class ReduceOp:
    SUM = "sum"
    AVG = "avg"
    MAX = "max"
    MIN = "min"
    ALL = (SUM, AVG, MAX, MIN)


_TORCH_OP = {ReduceOp.SUM: dist.ReduceOp.SUM, ReduceOp.AVG: dist.ReduceOp.SUM, ReduceOp.MAX: dist.ReduceOp.MAX,
             ReduceOp.MIN: dist.ReduceOp.MIN}


@dataclass
class CommunicationStats:
    calls: int = 0
    bytes: int = 0
    seconds: float = 0.0
    wait_seconds: float = 0.0

    def merge(self, other: CommunicationStats) -> None:
        self.calls += other.calls
        self.bytes += other.bytes
        self.seconds += other.seconds
        self.wait_seconds += other.wait_seconds

    def as_dict(self) -> dict[str, float]:
        return {"calls": float(self.calls), "bytes": float(self.bytes), "seconds": self.seconds,
                "wait_seconds": self.wait_seconds}


@dataclass
class CommunicationRecorder:
    """Per-``op/group`` counters; pass one as ``recorder=`` to any wrapper or wrapper class."""

    enabled: bool = True
    by_operation: dict[str, CommunicationStats] = field(default_factory=dict)

    def _slot(self, operation: str, group_name: str) -> CommunicationStats:
        return self.by_operation.setdefault(f"{operation}/{group_name}", CommunicationStats())

    def record(self, operation: str, group_name: str, *, num_bytes: int, seconds: float = 0.0, wait_seconds: float = 0.0) -> None:
        if self.enabled:
            slot = self._slot(operation, group_name)
            slot.calls += 1
            slot.bytes += num_bytes
            slot.seconds += seconds
            slot.wait_seconds += wait_seconds

    def record_wait(self, operation: str, group_name: str, *, wait_seconds: float) -> None:
        if self.enabled:
            self._slot(operation, group_name).wait_seconds += wait_seconds

    def total(self) -> CommunicationStats:
        out = CommunicationStats()
        for s in self.by_operation.values():
            out.merge(s)
        return out

    def reset(self) -> None:
        self.by_operation.clear()

    def summary(self) -> str:
        if not self.by_operation:
            return "nothing was communicated"
        lines = ["collectives by operation and group:"]
        for key in sorted(self.by_operation):
            s = self.by_operation[key]
            lines.append(f"  {key:<34} calls={s.calls:<6} MiB={s.bytes / 2**20:9.3f} launch_s={s.seconds:8.4f} "
                         f"wait_s={s.wait_seconds:8.4f}")
        return "\n".join(lines)


class AsyncWork:
    """Handle to an issued collective; ``wait()`` records wait time and runs an optional hook once."""

    __slots__ = ("_done", "_group_name", "_on_complete", "_operation", "_recorder", "_work")

    def __init__(self, work: Any, *, recorder: CommunicationRecorder | None = None, operation: str = "",
                 group_name: str = "", on_complete: Callable[[], None] | None = None) -> None:
        self._work = work
        self._recorder = recorder
        self._operation = operation
        self._group_name = group_name
        self._on_complete = on_complete
        self._done = work is None

    @property
    def is_completed(self) -> bool:
        return self._done or bool(self._work.is_completed())

    def wait(self) -> None:
        if not self._done:
            t0 = time.perf_counter()
            self._work.wait()
            if self._recorder is not None:
                self._recorder.record_wait(self._operation, self._group_name, wait_seconds=time.perf_counter() - t0)
            self._done = True
        if self._on_complete is not None:
            hook, self._on_complete = self._on_complete, None
            hook()


def _op(op: str, where: str, group: GroupHandle) -> Any:
    if op not in ReduceOp.ALL:
        raise CollectiveError(format_error(where, "this reduction is not supported", rank=group.global_rank,
                                           expected=list(ReduceOp.ALL), observed=op, resolution="use a ReduceOp constant"))
    return _TORCH_OP[op]


def _contiguous(tensor: torch.Tensor, where: str, group: GroupHandle) -> None:
    if not tensor.is_contiguous():
        raise CollectiveError(format_error(
            where, "collectives require contiguous tensors; some backends would silently copy a strided buffer",
            rank=group.global_rank, expected="a contiguous tensor",
            observed=f"shape={tuple(tensor.shape)} strides={tensor.stride()}", resolution="call .contiguous() first"))


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


_OBSERVERS: list[CommunicationRecorder] = []


@contextmanager
def observe_collectives(recorder: CommunicationRecorder | None = None) -> Iterator[CommunicationRecorder]:
    """Count every collective issued in this process while the block runs, whatever recorder its caller passed.

    Covers the wrappers of this module and the in-kernel NVLink collectives (DDP bucket
    all-reduce, FSDP reduce-scatter + AdamW and shard gathers, tensor-parallel GEMM collectives),
    which report through :func:`record_collective`.  Used to measure communication per step.
    """
    rec = recorder if recorder is not None else CommunicationRecorder()
    _OBSERVERS.append(rec)
    try:
        yield rec
    finally:
        _OBSERVERS.remove(rec)


def record_collective(recorder: CommunicationRecorder | None, operation: str, group_name: str, *, num_bytes: int,
                      seconds: float = 0.0) -> None:
    """Count one collective in ``recorder`` (if any) and in every active :func:`observe_collectives` block."""
    if recorder is not None:
        recorder.record(operation, group_name, num_bytes=num_bytes, seconds=seconds)
    for obs in _OBSERVERS:
        if obs is not recorder:
            obs.record(operation, group_name, num_bytes=num_bytes, seconds=seconds)


def _reduce_op_for(op: str, tensor: torch.Tensor, group: GroupHandle) -> tuple[Any, bool]:
    """(torch op, needs explicit pre-divide).  NCCL folds AVG's pre-divide into a pre-multiplied sum."""
    if op != ReduceOp.AVG:
        return _TORCH_OP[op], False
    if tensor.is_cuda and tensor.is_floating_point() and hasattr(dist, "_make_nccl_premul_sum"):
        return dist._make_nccl_premul_sum(1.0 / group.size), False
    return dist.ReduceOp.SUM, True


def all_reduce(tensor: torch.Tensor, group: GroupHandle, *, op: str = ReduceOp.SUM, async_op: bool = False,
               recorder: CommunicationRecorder | None = None) -> AsyncWork:
    """In-place all-reduce over ``group``."""
    where = "collectives.all_reduce"
    validate_group_membership(group, group.global_rank, where)
    _contiguous(tensor, where, group)
    _op(op, where, group)
    if group.is_trivial:
        return AsyncWork(None)
    t0 = time.perf_counter()
    torch_op, predivide = _reduce_op_for(op, tensor, group)
    if predivide:
        tensor.div_(group.size)
    work = dist.all_reduce(tensor, op=torch_op, group=group.process_group, async_op=async_op)
    record_collective(recorder, "all_reduce", group.name, num_bytes=_nbytes(tensor), seconds=time.perf_counter() - t0)
    return AsyncWork(work if async_op else None, recorder=recorder, operation="all_reduce", group_name=group.name)


def broadcast(tensor: torch.Tensor, group: GroupHandle, *, source_local_rank: int = 0, async_op: bool = False,
              recorder: CommunicationRecorder | None = None) -> AsyncWork:
    where = "collectives.broadcast"
    validate_group_membership(group, group.global_rank, where)
    _contiguous(tensor, where, group)
    if not 0 <= source_local_rank < group.size:
        raise CollectiveError(format_error(where, "the source index is not a position in the group", rank=group.global_rank,
                                           expected=f"0 <= r < {group.size}", observed=source_local_rank,
                                           resolution="give the position inside the group rather than the global rank"))
    if group.is_trivial:
        return AsyncWork(None)
    t0 = time.perf_counter()
    work = dist.broadcast(tensor, src=group.ranks[source_local_rank], group=group.process_group, async_op=async_op)
    record_collective(recorder, "broadcast", group.name, num_bytes=_nbytes(tensor), seconds=time.perf_counter() - t0)
    return AsyncWork(work if async_op else None, recorder=recorder, operation="broadcast", group_name=group.name)


def all_gather_tensor(tensor: torch.Tensor, group: GroupHandle, *, out: torch.Tensor | None = None,
                      recorder: CommunicationRecorder | None = None, async_op: bool = False) -> tuple[torch.Tensor, AsyncWork]:
    """Concatenate every member's tensor along dim 0 (rank order)."""
    where = "collectives.all_gather_tensor"
    validate_group_membership(group, group.global_rank, where)
    _contiguous(tensor, where, group)
    shape = (tensor.shape[0] * group.size, *tensor.shape[1:])
    if out is None:
        out = torch.empty(shape, dtype=tensor.dtype, device=tensor.device)
    elif tuple(out.shape) != shape:
        raise CollectiveError(format_error(where, "the output buffer is not shaped for this collective", rank=group.global_rank,
                                           expected=shape, observed=tuple(out.shape),
                                           resolution="allocate (members x rows, ...) for the gathered output"))
    if group.is_trivial:
        out.copy_(tensor)
        return out, AsyncWork(None)
    t0 = time.perf_counter()
    work = dist.all_gather_into_tensor(out, tensor, group=group.process_group, async_op=async_op)
    record_collective(recorder, "all_gather", group.name, num_bytes=_nbytes(tensor), seconds=time.perf_counter() - t0)
    return out, AsyncWork(work if async_op else None, recorder=recorder, operation="all_gather", group_name=group.name)


def reduce_scatter_tensor(tensor: torch.Tensor, group: GroupHandle, *, op: str = ReduceOp.SUM,
                          out: torch.Tensor | None = None, recorder: CommunicationRecorder | None = None,
                          async_op: bool = False) -> tuple[torch.Tensor, AsyncWork]:
    """Reduce over the group and keep this member's equal slice of dim 0."""
    where = "collectives.reduce_scatter_tensor"
    validate_group_membership(group, group.global_rank, where)
    _contiguous(tensor, where, group)
    _op(op, where, group)
    if tensor.shape[0] % group.size:
        raise CollectiveError(format_error(where, "dim 0 has to split into one equal block per group member",
                                           rank=group.global_rank, expected=f"shape[0] % {group.size} == 0",
                                           observed=tensor.shape[0], resolution="pad the buffer to a multiple of the group size"))
    shape = (tensor.shape[0] // group.size, *tensor.shape[1:])
    if out is None:
        out = torch.empty(shape, dtype=tensor.dtype, device=tensor.device)
    elif tuple(out.shape) != shape:
        raise CollectiveError(format_error(where, "the output buffer is not shaped for this collective", rank=group.global_rank,
                                           expected=shape, observed=tuple(out.shape),
                                           resolution="allocate (rows / members, ...) for the scattered output"))
    if group.is_trivial:
        out.copy_(tensor.view(shape))
        return out, AsyncWork(None)
    t0 = time.perf_counter()
    torch_op, predivide = _reduce_op_for(op, tensor, group)
    if predivide:
        tensor = tensor.div(group.size)
    work = dist.reduce_scatter_tensor(out, tensor, op=torch_op, group=group.process_group, async_op=async_op)
    record_collective(recorder, "reduce_scatter", group.name, num_bytes=_nbytes(tensor), seconds=time.perf_counter() - t0)
    return out, AsyncWork(work if async_op else None, recorder=recorder, operation="reduce_scatter", group_name=group.name)


def all_to_all_tensor(tensor: torch.Tensor, group: GroupHandle, *, recorder: CommunicationRecorder | None = None) -> torch.Tensor:
    """Equal-split all-to-all along dim 0 (chunk ``i`` goes to member ``i``)."""
    where = "collectives.all_to_all_tensor"
    validate_group_membership(group, group.global_rank, where)
    _contiguous(tensor, where, group)
    if tensor.shape[0] % group.size:
        raise CollectiveError(format_error(where, "dim 0 has to split into one equal block per group member",
                                           rank=group.global_rank, expected=f"shape[0] % {group.size} == 0",
                                           observed=tensor.shape[0], resolution="pad the leading dimension first"))
    if group.is_trivial:
        return tensor.clone()
    out = torch.empty_like(tensor)
    t0 = time.perf_counter()
    dist.all_to_all_single(out, tensor, group=group.process_group)
    record_collective(recorder, "all_to_all", group.name, num_bytes=_nbytes(tensor), seconds=time.perf_counter() - t0)
    return out


def _peer(group: GroupHandle, local: int, where: str, role: str) -> int:
    if not 0 <= local < group.size:
        raise CollectiveError(format_error(where, f"{role} outside the group", rank=group.global_rank,
                                           expected=f"0 <= r < {group.size}", observed=local, resolution="give the position inside the group"))
    peer = group.ranks[local]
    if peer == group.global_rank:
        raise CollectiveError(format_error(where, "a rank cannot exchange with itself; a blocking send/recv would deadlock",
                                           rank=group.global_rank, expected="a different rank", observed=peer,
                                           resolution="do not send a tensor to the rank that owns it"))
    return peer


def send_tensor(tensor: torch.Tensor, group: GroupHandle, *, destination_local_rank: int) -> None:
    where = "collectives.send_tensor"
    validate_group_membership(group, group.global_rank, where)
    _contiguous(tensor, where, group)
    dist.send(tensor, dst=_peer(group, destination_local_rank, where, "destination"), group=group.process_group)


def recv_tensor(tensor: torch.Tensor, group: GroupHandle, *, source_local_rank: int) -> torch.Tensor:
    where = "collectives.recv_tensor"
    validate_group_membership(group, group.global_rank, where)
    _contiguous(tensor, where, group)
    dist.recv(tensor, src=_peer(group, source_local_rank, where, "source"), group=group.process_group)
    return tensor


def all_gather_object_in_group(obj: Any, group: GroupHandle) -> list[Any]:
    validate_group_membership(group, group.global_rank, "collectives.all_gather_object")
    if group.is_trivial:
        return [obj]
    out: list[Any] = [None] * group.size
    dist.all_gather_object(out, obj, group=group.process_group)
    return out


def assert_metadata_consistent(payload: Any, group: GroupHandle, *, name: str, operation: str = "collectives.consistency") -> None:
    """Raise on every rank if ``payload`` differs anywhere in the group."""
    if group.is_trivial:
        return
    gathered = all_gather_object_in_group(payload, group)
    for local, value in enumerate(gathered):
        if value != gathered[0]:
            raise ParameterConsistencyError(format_error(
                operation, f"{name} differs across the {group.name!r} group; the collectives that follow would mismatch",
                rank=group.global_rank, expected=f"the group's first rank (global {group.ranks[0]}): {gathered[0]!r}",
                observed=f"local rank {local} (global {group.ranks[local]}): {value!r}",
                resolution="build the model identically on every rank of this group (same seed, config, module order)"))


def assert_tensor_consistent(tensor: torch.Tensor, group: GroupHandle, *, name: str, rtol: float = 0.0, atol: float = 0.0,
                             operation: str = "collectives.tensor_consistency") -> None:
    """Compare ``tensor`` with local rank 0's copy (broadcast) within tolerance."""
    if group.is_trivial:
        return
    reference = tensor.detach().clone().contiguous()
    broadcast(reference, group, source_local_rank=0).wait()
    if not torch.allclose(tensor.detach(), reference, rtol=rtol, atol=atol):
        delta = (tensor.detach().double() - reference.double()).abs().max().item()
        raise ParameterConsistencyError(format_error(
            operation, f"{name} is not the same here as on the group's first rank", rank=group.global_rank,
            expected=f"max |delta| <= {atol} (+ rtol {rtol})", observed=f"max |delta| = {delta:.3e}",
            resolution="seed identically on every rank and broadcast parameters at construction"))


def sum_scalar(value: float | torch.Tensor, group: GroupHandle, *, device: torch.device, op: str = ReduceOp.SUM,
               recorder: CommunicationRecorder | None = None) -> float:
    """All-reduce one scalar (fp64) and return it on the host."""
    if group.is_trivial:
        return float(value)
    buffer = torch.tensor([float(value)], dtype=torch.float64, device=device)
    all_reduce(buffer, group, op=op, recorder=recorder).wait()
    return float(buffer.item())


def concat_shard_sizes(numel: int, group_size: int) -> tuple[int, int]:
    """(padded total, per-rank shard) for an equal split with ceil division."""
    if group_size < 1:
        raise CollectiveError(format_error("collectives.concat_shard_sizes", "a group has at least one member", expected=">= 1",
                                           observed=group_size, resolution="give the number of members of the group"))
    shard = -(-numel // group_size)
    return shard * group_size, shard


def wait_all(works: Iterable[AsyncWork]) -> None:
    for work in works:
        work.wait()


def log_group_layout(groups: Sequence[GroupHandle]) -> None:
    for h in groups:
        _LOG.debug("%-16s %d ranks (this is #%d): %s", h.name, h.size, h.local_rank, h.ranks)
