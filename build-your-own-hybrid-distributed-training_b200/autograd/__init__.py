"""Differentiable collectives (forward collective + adjoint)."""

from .collectives import (
    all_gather_along_dim,
    copy_to_group,
    gather_from_group,
    gather_from_sequence_parallel_region,
    reduce_from_group,
    reduce_scatter_along_dim,
    reduce_scatter_to_group,
    scatter_to_group,
)

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
