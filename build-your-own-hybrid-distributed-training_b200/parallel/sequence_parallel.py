"""Sequence-parallel helpers: split/gather the sequence dimension with adjoints.

Behaviour of ``src/hybrid_training/parallel/sequence_parallel.py:103-453``:
uneven sequences are right-padded to a multiple of the group size (causal
masking makes the padded tail invisible to real positions), scattered, and
unpadded after the gather; norm layers run on sequence shards and their
parameters are marked as partial-gradient so the hybrid model sums them over
the sequence group.  :class:`SequenceParallelLayerNorm` (and the RMS variant)
run the fused norm kernel.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn

from .. import ops
from ..autograd.collectives import gather_from_group, reduce_scatter_to_group, scatter_to_group
from ..distributed.groups import GroupHandle
from ..errors import ShardingError, format_error

__all__ = [
    "SEQUENCE_DIM",
    "SequenceParallelLayerNorm",
    "SequenceParallelRMSNorm",
    "SequenceShardInfo",
    "gather_sequence",
    "local_sequence_slice",
    "pad_sequence_dimension",
    "reduce_scatter_sequence",
    "scatter_sequence",
    "unpad_sequence_dimension",
]

SEQUENCE_DIM = 1


@dataclass(frozen=True)
class SequenceShardInfo:
    original_length: int
    padded_length: int
    group_size: int
    local_length: int

    @classmethod
    def for_length(cls, length: int, group_size: int) -> SequenceShardInfo:
        if group_size < 1:
            raise ShardingError(format_error("sequence_parallel.SequenceShardInfo", "a group has at least one member",
                                             expected=">= 1", observed=group_size, resolution="give the number of sequence ranks"))
        padded = -(-length // group_size) * group_size
        return cls(length, padded, group_size, padded // group_size)

    @property
    def padding(self) -> int:
        return self.padded_length - self.original_length

    @property
    def requires_padding(self) -> bool:
        return self.padding > 0

    def local_range(self, local_rank: int) -> tuple[int, int]:
        start = local_rank * self.local_length
        return start, start + self.local_length


def pad_sequence_dimension(x: torch.Tensor, group_size: int, *, dim: int = SEQUENCE_DIM) -> tuple[torch.Tensor, SequenceShardInfo]:
    info = SequenceShardInfo.for_length(x.shape[dim], group_size)
    if not info.requires_padding:
        return x, info
    shape = list(x.shape)
    shape[dim] = info.padding
    return torch.cat([x, x.new_zeros(shape)], dim=dim), info


def unpad_sequence_dimension(x: torch.Tensor, info: SequenceShardInfo, *, dim: int = SEQUENCE_DIM) -> torch.Tensor:
    if x.shape[dim] != info.padded_length:
        raise ShardingError(format_error("sequence_parallel.unpad_sequence_dimension", "tensor does not have the padded length",
                                         expected=info.padded_length, observed=x.shape[dim],
                                         resolution="pass the SequenceShardInfo that produced the padding"))
    return x.narrow(dim, 0, info.original_length) if info.requires_padding else x


def _require_divisible(x: torch.Tensor, group: GroupHandle, dim: int, op: str) -> None:
    if x.shape[dim] % group.size:
        raise ShardingError(format_error(op, "the sequence length does not split evenly over the sequence ranks",
                                         rank=group.global_rank, expected=f"{x.shape[dim]} % {group.size} == 0",
                                         observed=x.shape[dim] % group.size,
                                         resolution="pad with pad_sequence_dimension() first"))


def scatter_sequence(x: torch.Tensor, group: GroupHandle, *, dim: int = SEQUENCE_DIM) -> torch.Tensor:
    _require_divisible(x, group, dim, "sequence_parallel.scatter_sequence")
    return scatter_to_group(x, group, dim=dim)


def gather_sequence(x: torch.Tensor, group: GroupHandle, *, dim: int = SEQUENCE_DIM) -> torch.Tensor:
    return gather_from_group(x, group, dim=dim)


def reduce_scatter_sequence(x: torch.Tensor, group: GroupHandle, *, dim: int = SEQUENCE_DIM) -> torch.Tensor:
    _require_divisible(x, group, dim, "sequence_parallel.reduce_scatter_sequence")
    return reduce_scatter_to_group(x, group, dim=dim)


def local_sequence_slice(total_length: int, group: GroupHandle) -> tuple[int, int]:
    if total_length % group.size:
        raise ShardingError(format_error("sequence_parallel.local_sequence_slice", "sequence length not divisible by the SP size",
                                         rank=group.global_rank, expected=f"{total_length} % {group.size} == 0",
                                         observed=total_length % group.size, resolution="pad the sequence first"))
    local = total_length // group.size
    return group.local_rank * local, (group.local_rank + 1) * local


def _mark_norm(params: list[nn.Parameter], group: GroupHandle | None, sequence_parallel: bool) -> None:
    if group is None:
        return
    from .tensor_parallel import _mark_replicated, mark_sequence_parallel_partial

    for p in params:
        _mark_replicated(p, group)
        if sequence_parallel:
            mark_sequence_parallel_partial(p)


class SequenceParallelLayerNorm(nn.Module):
    """LayerNorm over the hidden dimension of a (possibly sequence-sharded) activation."""

    def __init__(self, hidden_size: int, *, eps: float = 1e-5, group: GroupHandle | None = None,
                 sequence_parallel: bool = False, device: torch.device | None = None, dtype: torch.dtype | None = None) -> None:
        super().__init__()
        self.hidden_size, self.eps, self.sequence_parallel = hidden_size, eps, sequence_parallel
        self.weight = nn.Parameter(torch.ones(hidden_size, device=device, dtype=dtype))
        self.bias = nn.Parameter(torch.zeros(hidden_size, device=device, dtype=dtype))
        _mark_norm([self.weight, self.bias], group, sequence_parallel)

    def forward(self, x: torch.Tensor, delta: torch.Tensor | None = None, out_dtype: torch.dtype | None = None):
        """``norm(x)``; with ``delta`` returns ``(x + delta, norm(x + delta))`` (fused residual add)."""
        r, y = ops.add_norm(x, delta, self.weight, self.bias, eps=self.eps, rms=False, out_dtype=out_dtype)
        return y if delta is None else (r, y)

    def extra_repr(self) -> str:
        return f"hidden_size={self.hidden_size}, eps={self.eps}, sequence_parallel={self.sequence_parallel}"


class SequenceParallelRMSNorm(nn.Module):
    """RMSNorm (no bias) over the hidden dimension of a (possibly sequence-sharded) activation."""

    def __init__(self, hidden_size: int, *, eps: float = 1e-5, group: GroupHandle | None = None,
                 sequence_parallel: bool = False, device: torch.device | None = None, dtype: torch.dtype | None = None) -> None:
        super().__init__()
        self.hidden_size, self.eps, self.sequence_parallel = hidden_size, eps, sequence_parallel
        self.weight = nn.Parameter(torch.ones(hidden_size, device=device, dtype=dtype))
        _mark_norm([self.weight], group, sequence_parallel)

    def forward(self, x: torch.Tensor, delta: torch.Tensor | None = None, out_dtype: torch.dtype | None = None):
        r, y = ops.add_norm(x, delta, self.weight, None, eps=self.eps, rms=True, out_dtype=out_dtype)
        return y if delta is None else (r, y)

    def extra_repr(self) -> str:
        return f"hidden_size={self.hidden_size}, eps={self.eps}, sequence_parallel={self.sequence_parallel}"
