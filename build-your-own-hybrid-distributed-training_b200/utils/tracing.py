"""NVTX ranges around the framework's phases and fused collectives, for profiler timelines.

The reference has no tracing beyond its communication recorder
(``src/hybrid_training/distributed/collectives.py:97-231``).  Here every phase that a timeline
reader needs to find -- the forward / backward / optimizer parts of a step, each DDP bucket
reduction, each FSDP gather and fused reduce-scatter, each fused tensor-parallel GEMM -- is
wrapped in a named NVTX range.  Ranges are off by default (zero cost beyond one boolean test);
``HT_NVTX=1`` in the environment or :func:`set_tracing` turns them on.  NVTX pushes are host
calls, so a range inside a captured CUDA graph marks the capture, not each replay.
"""

from __future__ import annotations

import os
from collections.abc import Iterator
from contextlib import contextmanager

import torch

__all__ = ["set_tracing", "trace_range", "tracing_enabled"]

_ENABLED = os.environ.get("HT_NVTX", "0") == "1"


def set_tracing(enabled: bool) -> None:
    """Turn NVTX ranges on or off for this process."""
    global _ENABLED
    _ENABLED = bool(enabled)


def tracing_enabled() -> bool:
    return _ENABLED and torch.cuda.is_available()


@contextmanager
def trace_range(name: str) -> Iterator[None]:
    """``with trace_range("ddp/bucket 3"): ...`` -- a named NVTX range when tracing is on."""
    if not (_ENABLED and torch.cuda.is_available()):
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
