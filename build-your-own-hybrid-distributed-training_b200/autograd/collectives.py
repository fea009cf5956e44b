"""Differentiable collectives: each forward collective paired with its adjoint.

=============================  =======================  ========================
function                       forward                  backward
=============================  =======================  ========================
``copy_to_group``  (f)         identity                 all-reduce
``reduce_from_group`` (g)      all-reduce               identity
``gather_from_group``          all-gather along dim     keep own slice
``scatter_to_group``           keep own slice           all-gather along dim
``reduce_scatter_to_group``    reduce-scatter on dim    all-gather along dim
``gather_from_sequence_        all-gather on dim        reduce-scatter on dim
parallel_region``
=============================  =======================  ========================

These are the adjoints of ``src/hybrid_training/autograd/collectives.py:166-420``.
The sequence-parallel gather's adjoint is a *reduce-scatter*, not a slice:
every rank's column-parallel layer consumed the full gathered sequence, so the
gradient of each position is the sum of all ranks' contributions.  The fused
paths in :mod:`hybrid_training.ops.comm` implement the same adjoints with the
collective inside the GEMM (all-gather in its operand loads, reduce-scatter in
its epilogue) or in an NVLink all-reduce kernel that reads the GEMM's output
from peer memory.
"""

from __future__ import annotations

from typing import Any

import torch

from ..distributed.collectives import CommunicationRecorder, ReduceOp, all_gather_tensor, all_reduce, reduce_scatter_tensor
from ..distributed.groups import GroupHandle
from ..errors import CollectiveError, format_error
from ..utils.tensors import split_tensor_along_dim

__all__ = [
    "all_gather_along_dim",
    "copy_to_group",
    "gather_from_group",
    "gather_from_sequence_parallel_region",
    "reduce_from_group",
    "reduce_scatter_along_dim",
    "reduce_scatter_to_group",
    "scatter_to_group",
]


def all_gather_along_dim(tensor: torch.Tensor, group: GroupHandle, dim: int, *,
                         recorder: CommunicationRecorder | None = None) -> torch.Tensor:
    """All-gather ``tensor`` and concatenate the pieces along ``dim`` (rank order)."""
    if group.is_trivial:
        return tensor
    dim %= tensor.dim()
    if dim == 0:
        out, work = all_gather_tensor(tensor.contiguous(), group, recorder=recorder)
        work.wait()
        return out
    moved = tensor.movedim(dim, 0).contiguous()
    out, work = all_gather_tensor(moved, group, recorder=recorder)
    work.wait()
    return out.movedim(0, dim).contiguous()


def reduce_scatter_along_dim(tensor: torch.Tensor, group: GroupHandle, dim: int, *, op: str = ReduceOp.SUM,
                             recorder: CommunicationRecorder | None = None) -> torch.Tensor:
    """Sum over the group, keep this rank's equal slice of ``dim``."""
    if group.is_trivial:
        return tensor
    dim %= tensor.dim()
    if tensor.shape[dim] % group.size:
        raise CollectiveError(format_error(
            "autograd.reduce_scatter_along_dim", f"dimension {dim} has to split evenly over the group",
            rank=group.global_rank, expected=f"{tensor.shape[dim]} % {group.size} == 0",
            observed=tensor.shape[dim] % group.size, resolution="pad the dimension or choose a dividing parallel size"))
    moved = tensor.movedim(dim, 0).contiguous()
    out, work = reduce_scatter_tensor(moved, group, op=op, recorder=recorder)
    work.wait()
    return out if dim == 0 else out.movedim(0, dim).contiguous()


class _CopyToGroup(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, tensor: torch.Tensor, group: GroupHandle) -> torch.Tensor:
        ctx.group = group
        return tensor

    @staticmethod
    def backward(ctx: Any, grad: torch.Tensor) -> tuple[torch.Tensor, None]:
        if ctx.group.is_trivial:
            return grad, None
        grad = grad.contiguous()
        all_reduce(grad, ctx.group, op=ReduceOp.SUM).wait()
        return grad, None


class _ReduceFromGroup(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, tensor: torch.Tensor, group: GroupHandle) -> torch.Tensor:
        if group.is_trivial:
            return tensor
        out = tensor.contiguous().clone()
        all_reduce(out, group, op=ReduceOp.SUM).wait()
        return out

    @staticmethod
    def backward(ctx: Any, grad: torch.Tensor) -> tuple[torch.Tensor, None]:
        return grad, None


class _GatherFromGroup(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, tensor: torch.Tensor, group: GroupHandle, dim: int) -> torch.Tensor:
        ctx.group, ctx.dim = group, dim % tensor.dim()
        return all_gather_along_dim(tensor, group, ctx.dim)

    @staticmethod
    def backward(ctx: Any, grad: torch.Tensor) -> tuple[torch.Tensor, None, None]:
        if ctx.group.is_trivial:
            return grad, None, None
        return split_tensor_along_dim(grad, ctx.dim, ctx.group.size)[ctx.group.local_rank], None, None


class _ScatterToGroup(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, tensor: torch.Tensor, group: GroupHandle, dim: int) -> torch.Tensor:
        ctx.group, ctx.dim = group, dim % tensor.dim()
        if group.is_trivial:
            return tensor
        return split_tensor_along_dim(tensor, ctx.dim, group.size)[group.local_rank]

    @staticmethod
    def backward(ctx: Any, grad: torch.Tensor) -> tuple[torch.Tensor, None, None]:
        if ctx.group.is_trivial:
            return grad, None, None
        return all_gather_along_dim(grad.contiguous(), ctx.group, ctx.dim), None, None


class _ReduceScatterToGroup(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, tensor: torch.Tensor, group: GroupHandle, dim: int) -> torch.Tensor:
        ctx.group, ctx.dim = group, dim % tensor.dim()
        return reduce_scatter_along_dim(tensor, group, ctx.dim, op=ReduceOp.SUM)

    @staticmethod
    def backward(ctx: Any, grad: torch.Tensor) -> tuple[torch.Tensor, None, None]:
        if ctx.group.is_trivial:
            return grad, None, None
        return all_gather_along_dim(grad.contiguous(), ctx.group, ctx.dim), None, None


class _GatherFromSequenceParallelRegion(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, tensor: torch.Tensor, group: GroupHandle, dim: int) -> torch.Tensor:
        ctx.group, ctx.dim = group, dim % tensor.dim()
        return all_gather_along_dim(tensor, group, ctx.dim)

    @staticmethod
    def backward(ctx: Any, grad: torch.Tensor) -> tuple[torch.Tensor, None, None]:
        if ctx.group.is_trivial:
            return grad, None, None
        return reduce_scatter_along_dim(grad.contiguous(), ctx.group, ctx.dim, op=ReduceOp.SUM), None, None


def copy_to_group(tensor: torch.Tensor, group: GroupHandle) -> torch.Tensor:
    """Identity forward, all-reduce backward (Megatron ``f``)."""
    return _CopyToGroup.apply(tensor, group)


def reduce_from_group(tensor: torch.Tensor, group: GroupHandle) -> torch.Tensor:
    """All-reduce forward, identity backward (Megatron ``g``)."""
    return _ReduceFromGroup.apply(tensor, group)


def gather_from_group(tensor: torch.Tensor, group: GroupHandle, dim: int = -1) -> torch.Tensor:
    return _GatherFromGroup.apply(tensor, group, dim)


def scatter_to_group(tensor: torch.Tensor, group: GroupHandle, dim: int = -1) -> torch.Tensor:
    return _ScatterToGroup.apply(tensor, group, dim)


def reduce_scatter_to_group(tensor: torch.Tensor, group: GroupHandle, dim: int = 1) -> torch.Tensor:
    return _ReduceScatterToGroup.apply(tensor, group, dim)


def gather_from_sequence_parallel_region(tensor: torch.Tensor, group: GroupHandle, dim: int = 1) -> torch.Tensor:
    """All-gather forward, reduce-scatter backward (entry to a column-parallel layer under SP)."""
    return _GatherFromSequenceParallelRegion.apply(tensor, group, dim)
