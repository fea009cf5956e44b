"""Analytic memory model and measured memory snapshots.

Parity with ``src/hybrid_training/utils/memory.py:148-369``: the analytic
model counts persistent parameters, gradients and optimizer slots per rank
(``P/G`` each under sharding) plus the transient gathered unit; the snapshot
reads the CUDA caching allocator (or scans live tensors on CPU).
"""

from __future__ import annotations

import gc
from collections.abc import Iterable
from dataclasses import dataclass, field

import torch

__all__ = [
    "MemoryEstimate",
    "MemorySnapshot",
    "capture_memory",
    "estimate_training_memory",
    "format_bytes",
    "module_parameter_bytes",
    "reset_peak_memory",
    "tensor_inventory",
]

OPTIMIZER_STATE_SLOTS: dict[str, int] = {"adamw": 2, "adam": 2, "sgd": 0, "sgd_momentum": 1}


def format_bytes(num_bytes: float) -> str:
    value = float(num_bytes)
    if abs(value) < 1024:
        return f"{value:.0f} B"
    for unit in ("KiB", "MiB", "GiB", "TiB"):
        value /= 1024.0
        if abs(value) < 1024.0 or unit == "TiB":
            return f"{value:.2f} {unit}"
    return f"{value:.2f} TiB"


@dataclass(frozen=True)
class MemoryEstimate:
    persistent_parameters: int
    gradients: int
    optimizer_state: int
    transient_gathered_parameters: int = 0
    transient_gathered_gradients: int = 0

    @property
    def steady_state(self) -> int:
        return self.persistent_parameters + self.gradients + self.optimizer_state

    @property
    def peak(self) -> int:
        return self.steady_state + self.transient_gathered_parameters + self.transient_gathered_gradients

    def as_dict(self) -> dict[str, int]:
        return {
            "persistent_parameters": self.persistent_parameters,
            "gradients": self.gradients,
            "optimizer_state": self.optimizer_state,
            "transient_gathered_parameters": self.transient_gathered_parameters,
            "transient_gathered_gradients": self.transient_gathered_gradients,
            "steady_state": self.steady_state,
            "peak": self.peak,
        }

    def report(self) -> str:
        return "\n".join(f"  {k.replace('_', ' '):<30} {format_bytes(v):>12}" for k, v in self.as_dict().items())


def estimate_training_memory(
    total_parameters: int,
    *,
    shard_group_size: int = 1,
    largest_unit_parameters: int | None = None,
    optimizer: str = "adamw",
    parameter_bytes: int = 4,
    gradient_bytes: int = 4,
    optimizer_state_bytes: int = 4,
    reshard_after_forward: bool = True,
) -> MemoryEstimate:
    """Bytes per rank for parameters, gradients and optimizer state under flat sharding."""
    if shard_group_size < 1:
        raise ValueError(f"the shard group has at least one rank; got {shard_group_size}")
    if optimizer not in OPTIMIZER_STATE_SLOTS:
        raise ValueError(f"no state-size rule for optimizer {optimizer!r} (known: {', '.join(sorted(OPTIMIZER_STATE_SLOTS))})")
    unit = total_parameters if largest_unit_parameters is None else largest_unit_parameters
    local = -(-total_parameters // shard_group_size)
    gathered_params = gathered_grads = 0
    if shard_group_size > 1:
        gathered_params = unit * parameter_bytes * (1 if reshard_after_forward else 2)
        gathered_grads = unit * gradient_bytes
    return MemoryEstimate(
        persistent_parameters=local * parameter_bytes,
        gradients=local * gradient_bytes,
        optimizer_state=local * OPTIMIZER_STATE_SLOTS[optimizer] * optimizer_state_bytes,
        transient_gathered_parameters=gathered_params,
        transient_gathered_gradients=gathered_grads,
    )


@dataclass
class MemorySnapshot:
    device: torch.device
    allocated_bytes: int = 0
    reserved_bytes: int = 0
    peak_allocated_bytes: int = 0
    live_tensor_bytes: int = 0
    source: str = "gc"
    extra: dict[str, int] = field(default_factory=dict)

    def report(self) -> str:
        rows = [("allocated", self.allocated_bytes), ("reserved", self.reserved_bytes),
                ("peak allocated", self.peak_allocated_bytes), ("live tensors (gc)", self.live_tensor_bytes),
                *sorted(self.extra.items())]
        return "\n".join([f"memory on {self.device} (source={self.source}):"] +
                         [f"  {k:<20} {format_bytes(v):>12}" for k, v in rows])


def _live_tensor_bytes(device: torch.device) -> int:
    seen: set[int] = set()
    total = 0
    for obj in gc.get_objects():
        try:
            if not torch.is_tensor(obj) or obj.device != device:
                continue
            storage = obj.untyped_storage()
            if storage.data_ptr() in seen:
                continue
            seen.add(storage.data_ptr())
            total += storage.nbytes()
        except (ReferenceError, RuntimeError):
            continue
    return total


def capture_memory(device: torch.device, *, include_gc_scan: bool = False) -> MemorySnapshot:
    if device.type == "cuda" and torch.cuda.is_available():
        torch.cuda.synchronize(device)
        snap = MemorySnapshot(device, int(torch.cuda.memory_allocated(device)), int(torch.cuda.memory_reserved(device)),
                              int(torch.cuda.max_memory_allocated(device)), source="cuda")
        if include_gc_scan:
            snap.live_tensor_bytes = _live_tensor_bytes(device)
        return snap
    live = _live_tensor_bytes(device)
    return MemorySnapshot(device, allocated_bytes=live, live_tensor_bytes=live, source="gc")


def reset_peak_memory(device: torch.device) -> None:
    if device.type == "cuda" and torch.cuda.is_available():
        torch.cuda.reset_peak_memory_stats(device)


def tensor_inventory(tensors: Iterable[torch.Tensor]) -> dict[str, int]:
    out: dict[str, int] = {}
    for t in tensors:
        out[str(t.dtype)] = out.get(str(t.dtype), 0) + t.numel() * t.element_size()
    return out


def module_parameter_bytes(module: torch.nn.Module) -> dict[str, int]:
    params = list(module.parameters())
    return {
        "parameters": sum(p.numel() * p.element_size() for p in params),
        "gradients": sum(p.grad.numel() * p.grad.element_size() for p in params if p.grad is not None),
        "buffers": sum(b.numel() * b.element_size() for b in module.buffers()),
    }
