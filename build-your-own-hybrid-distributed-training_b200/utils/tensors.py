"""Flat-buffer layout arithmetic: the core of FSDP sharding, DDP buckets and resharding.

Parity with the reference's ``src/hybrid_training/utils/tensors.py:58-532``:
``FlatEntry`` / ``ShardRange`` records, layout building, flatten/unflatten,
padding to a multiple, equal shard ranges (ceil division, last shard padded)
and interval intersection.  The flat layout is the same (tensors concatenated
in registration order, padding at the end) because the checkpoint manifest
expresses shards as intervals of exactly that layout.
"""

from __future__ import annotations

from collections.abc import Iterable, Sequence
from dataclasses import dataclass

import torch

from ..errors import ShardingError, format_error

__all__ = [
    "FlatEntry",
    "ShardRange",
    "build_flat_layout",
    "bytes_of",
    "even_shard_ranges",
    "flatten_dense_tensors",
    "intersect_ranges",
    "numel_of",
    "pad_flat_tensor",
    "shard_range_for",
    "split_tensor_along_dim",
    "unflatten_to_views",
]


def _err(op: str, problem: str, expected: object, observed: object, fix: str) -> ShardingError:
    return ShardingError(format_error(f"tensors.{op}", problem, expected=expected, observed=observed, resolution=fix))


@dataclass(frozen=True)
class FlatEntry:
    """Where one named tensor lives inside a flat buffer."""

    name: str
    shape: tuple[int, ...]
    offset: int
    numel: int
    dtype_str: str
    requires_grad: bool = True

    @property
    def end(self) -> int:
        return self.offset + self.numel

    def as_dict(self) -> dict[str, object]:
        return {"name": self.name, "shape": list(self.shape), "offset": self.offset, "numel": self.numel,
                "dtype": self.dtype_str, "requires_grad": self.requires_grad}


@dataclass(frozen=True)
class ShardRange:
    """Elements ``start`` up to (not including) ``start + length`` of a 1-D buffer."""

    start: int
    length: int

    def __post_init__(self) -> None:
        if self.start < 0 or self.length < 0:
            raise _err("ShardRange", "a shard range cannot start or extend below zero", "non-negative start and length",
                       f"start={self.start}, length={self.length}", "recompute the offsets")

    @property
    def end(self) -> int:
        return self.start + self.length

    @property
    def is_empty(self) -> bool:
        return self.length == 0

    def as_tuple(self) -> tuple[int, int]:
        return (self.start, self.length)


def build_flat_layout(named_tensors: Sequence[tuple[str, torch.Tensor]]) -> tuple[tuple[FlatEntry, ...], int]:
    """Concatenate tensors in order; returns the entries and the total element count."""
    if not named_tensors:
        raise _err("build_flat_layout", "there is nothing to flatten", ">= 1 tensor", 0,
                   "do not create a flat buffer for a module with no parameters")
    entries: list[FlatEntry] = []
    names: set[str] = set()
    cursor = 0
    for name, tensor in named_tensors:
        if name in names:
            raise _err("build_flat_layout", "duplicate tensor name in one flat buffer (a tied tensor registered twice)",
                       "unique names", name, "list each shared (tied) tensor once")
        names.add(name)
        n = tensor.numel()
        entries.append(FlatEntry(name, tuple(tensor.shape), cursor, n, str(tensor.dtype), bool(tensor.requires_grad)))
        cursor += n
    return tuple(entries), cursor


def flatten_dense_tensors(tensors: Iterable[torch.Tensor], *, out: torch.Tensor | None = None) -> torch.Tensor:
    """Copy tensors of one dtype/device back to back into a 1-D buffer."""
    items = list(tensors)
    if not items:
        raise _err("flatten_dense_tensors", "nothing to flatten", ">= 1 tensor", 0, "give one or more tensors")
    dtype, device = items[0].dtype, items[0].device
    for t in items:
        if t.dtype != dtype or t.device != device:
            raise _err("flatten_dense_tensors", "one flat buffer holds one dtype on one device",
                       f"{dtype} on {device}", f"{t.dtype} on {t.device}", "group tensors by dtype/device first")
    total = sum(t.numel() for t in items)
    if out is None:
        out = torch.empty(total, dtype=dtype, device=device)
    elif out.numel() != total:
        raise _err("flatten_dense_tensors", "the output buffer has the wrong number of elements", total, out.numel(),
                   "allocate exactly the total element count")
    cursor = 0
    for t in items:
        out[cursor:cursor + t.numel()].copy_(t.detach().reshape(-1))
        cursor += t.numel()
    return out


def unflatten_to_views(flat: torch.Tensor, entries: Sequence[FlatEntry]) -> list[torch.Tensor]:
    """Shaped views into ``flat`` for each entry (no copies)."""
    if flat.dim() != 1:
        raise _err("unflatten_to_views", "a flat buffer has a single dimension", "dim() == 1", flat.dim(),
                   "reshape to (-1,) first")
    need = entries[-1].end if entries else 0
    if flat.numel() < need:
        raise _err("unflatten_to_views", "the flat buffer holds fewer elements than the layout needs", f">= {need} elements", flat.numel(),
                   "size the buffer by the padded total")
    return [flat[e.offset:e.end].view(e.shape) for e in entries]


def pad_flat_tensor(flat: torch.Tensor, multiple: int, *, value: float = 0.0) -> torch.Tensor:
    """Right-pad a 1-D tensor to a multiple of ``multiple`` (returns it unchanged if aligned)."""
    if flat.dim() != 1:
        raise _err("pad_flat_tensor", "this needs a 1-D tensor", "dim() == 1", flat.dim(), "flatten first")
    if multiple < 1:
        raise _err("pad_flat_tensor", "padding rounds up to a multiple that is at least 1", ">= 1", multiple, "pass the group size")
    short = (-flat.numel()) % multiple
    if short == 0:
        return flat
    return torch.cat([flat, flat.new_full((short,), value)])


def even_shard_ranges(total_numel: int, num_shards: int) -> tuple[ShardRange, ...]:
    """``num_shards`` equal ranges of ``ceil(total / num_shards)`` elements (the last covers padding)."""
    if num_shards < 1:
        raise _err("even_shard_ranges", "a tensor is split into one or more shards", ">= 1", num_shards, "give the number of shard ranks")
    size = -(-total_numel // num_shards)
    return tuple(ShardRange(i * size, size) for i in range(num_shards))


def shard_range_for(total_numel: int, num_shards: int, shard_index: int) -> ShardRange:
    if not 0 <= shard_index < num_shards:
        raise _err("shard_range_for", "the shard index is not below the number of shards", f"0 <= i < {num_shards}", shard_index,
                   "give the position of the rank in the shard group")
    size = -(-total_numel // num_shards)
    return ShardRange(shard_index * size, size)


def intersect_ranges(a: ShardRange, b: ShardRange) -> ShardRange | None:
    """Overlap of two ranges, or ``None`` when they are disjoint."""
    lo, hi = max(a.start, b.start), min(a.end, b.end)
    return ShardRange(lo, hi - lo) if hi > lo else None


def split_tensor_along_dim(tensor: torch.Tensor, dim: int, num_parts: int, *, contiguous: bool = True) -> tuple[torch.Tensor, ...]:
    """Split ``dim`` into ``num_parts`` equal chunks (error if not divisible)."""
    if num_parts < 1:
        raise _err("split_tensor_along_dim", "a split has one or more parts", ">= 1", num_parts, "pass the group size")
    if not -tensor.dim() <= dim < tensor.dim():
        raise _err("split_tensor_along_dim", "the tensor has no such dimension", f"-{tensor.dim()} <= dim < {tensor.dim()}",
                   dim, "count the dimensions of the tensor")
    dim %= tensor.dim()
    size = tensor.shape[dim]
    if size % num_parts:
        raise _err("split_tensor_along_dim", f"{num_parts} equal parts do not tile dimension {dim} (size {size})",
                   f"{size} % {num_parts} == 0", size % num_parts, "pick a parallel size that divides the dimension")
    parts = torch.chunk(tensor, num_parts, dim=dim) if size else tuple(tensor for _ in range(num_parts))
    return tuple(p.contiguous() for p in parts) if contiguous else tuple(parts)


def numel_of(named_tensors: Iterable[tuple[str, torch.Tensor]]) -> int:
    return sum(t.numel() for _, t in named_tensors)


def bytes_of(tensors: Iterable[torch.Tensor]) -> int:
    return sum(t.numel() * t.element_size() for t in tensors)
