"""Collectives computed inside native kernels over NVLink peer memory.

``bucket_all_reduce`` averages one DDP gradient bucket across the data-parallel
group with a single kernel that reads the peers' buffers directly (two-shot
reduce-scatter + all-gather over P2P loads, or, when the NVLink switch offers
a multicast address and ``HT_NVLS=1``, one ``multimem.ld_reduce`` /
``multimem.st`` pass), folding the ``1/G`` scale into the reduction.  Its
input must live in a :class:`~hybrid_training.distributed.symmetric.SymmetricWorkspace`
allocation (DDP allocates its flat gradient buffer there).  Every wait in the
kernel is bounded; a timeout sets the workspace status word, which
``SymmetricWorkspace.check_status`` turns into a :class:`KernelError`.

The tensor-parallel fused paths (all-gather inside the first GEMM of a
column-parallel layer, reduce-scatter inside the GEMM of a row-parallel layer)
are exposed as :func:`all_gather_linear` / :func:`linear_reduce_scatter`;
:data:`HAS_FUSED_TENSOR_PARALLEL` tells the layers whether to use them.
"""

from __future__ import annotations

import os
from typing import Any

import torch

from ._ext import extension

__all__ = ["HAS_FUSED_TENSOR_PARALLEL", "all_gather_linear", "bucket_all_reduce", "linear_reduce_scatter"]

HAS_FUSED_TENSOR_PARALLEL = False
_TIMEOUT_S = float(os.environ.get("HT_COLLECTIVE_TIMEOUT_S", "30"))


def _slots(handle: Any, world: int) -> tuple[int, int]:
    """(first signal-pad slot used here, max blocks): the upper half of each pad is reserved for these kernels."""
    slots = int(handle.signal_pad_size) // 4
    base = slots // 2
    return base, max(1, (slots - base) // world)


def bucket_all_reduce(workspace: Any, flat: torch.Tensor, start: int, numel: int, scale: float) -> torch.Tensor:
    """Average ``flat[start:start+numel]`` over the workspace's group in place; returns the status tensor."""
    handle = workspace.handle_of(flat)
    world = workspace.group.size
    base, max_blocks = _slots(handle, world)
    mc = int(handle.multicast_ptr) if os.environ.get("HT_NVLS", "0") == "1" else 0
    extension().bucket_all_reduce(flat, list(handle.buffer_ptrs), list(handle.signal_pad_ptrs), mc, int(start), int(numel),
                                  float(scale), int(handle.rank), base, min(max_blocks, 64), workspace.status, _TIMEOUT_S)
    return workspace.status


def all_gather_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, workspace: Any, group: Any, *,
                      activation: str | None = None) -> torch.Tensor:
    raise NotImplementedError("fused all-gather GEMM is not available in this build")


def linear_reduce_scatter(x: torch.Tensor, weight: torch.Tensor, workspace: Any, group: Any) -> torch.Tensor:
    raise NotImplementedError("fused GEMM reduce-scatter is not available in this build")
