"""Seeding, seed derivation and RNG state capture/restore.

Behaviour follows the reference (``src/hybrid_training/utils/reproducibility.py:78-332``):
named seed streams, a ``temporary_seed`` context used to draw a full weight
matrix and keep one tensor-parallel slice (so every TP width initialises the
same global matrix), and RNG snapshots that serialise to tensors plus JSON
metadata for the checkpoint.  The stream hash here is BLAKE2b, not the
reference's string hash, so seeds are stable across processes and Python
versions without reproducing its mixing constants.
"""

from __future__ import annotations

import hashlib
import os
import random
from collections.abc import Iterator
from contextlib import contextmanager
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from ..logging import get_logger

__all__ = [
    "RngSnapshot",
    "capture_rng_state",
    "derive_seed",
    "restore_rng_state",
    "rng_state_from_serialisable",
    "rng_state_to_serialisable",
    "seed_everything",
    "temporary_seed",
]

_LOG = get_logger(__name__)


def derive_seed(base_seed: int, stream: str, index: int = 0) -> int:
    """Deterministic 31-bit seed for ``(base_seed, stream, index)``."""
    digest = hashlib.blake2b(f"{int(base_seed)}|{stream}|{int(index)}".encode(), digest_size=8).digest()
    return int.from_bytes(digest, "little") & 0x7FFFFFFF


@dataclass
class RngSnapshot:
    python_state: Any
    numpy_state: Any
    torch_cpu_state: torch.Tensor
    torch_cuda_states: list[torch.Tensor] | None = None


def capture_rng_state(*, include_cuda: bool = True) -> RngSnapshot:
    cuda = None
    if include_cuda and torch.cuda.is_available():
        cuda = [s.clone() for s in torch.cuda.get_rng_state_all()]
    return RngSnapshot(random.getstate(), np.random.get_state(), torch.get_rng_state().clone(), cuda)


def restore_rng_state(snapshot: RngSnapshot) -> None:
    random.setstate(snapshot.python_state)
    np.random.set_state(snapshot.numpy_state)
    torch.set_rng_state(snapshot.torch_cpu_state.to(torch.uint8).cpu())
    states = snapshot.torch_cuda_states
    if states is not None and torch.cuda.is_available():
        if torch.cuda.device_count() >= len(states):
            torch.cuda.set_rng_state_all([s.to(torch.uint8).cpu() for s in states])
        else:
            _LOG.warning("%d CUDA RNG states saved but %d device(s) visible; CUDA RNG not restored",
                         len(states), torch.cuda.device_count())


def seed_everything(seed: int, *, stream: str = "global", index: int = 0, deterministic: bool = True,
                    warn_only: bool = True) -> int:
    """Seed python/numpy/torch from a derived stream seed; optionally request deterministic kernels."""
    derived = derive_seed(seed, stream, index)
    random.seed(derived)
    np.random.seed(derived % 2**32)
    torch.manual_seed(derived)
    if deterministic:
        torch.backends.cudnn.benchmark = False
        torch.backends.cudnn.deterministic = True
        torch.use_deterministic_algorithms(True, warn_only=warn_only)
        os.environ.setdefault("CUBLAS_WORKSPACE_CONFIG", ":4096:8")
    return derived


@contextmanager
def temporary_seed(seed: int, *, devices: list[torch.device] | None = None) -> Iterator[None]:
    """Run a block under ``seed`` and restore every generator afterwards."""
    snapshot = capture_rng_state()
    try:
        random.seed(seed)
        np.random.seed(seed % 2**32)
        torch.manual_seed(seed)
        if devices:
            for device in devices:
                with torch.cuda.device(device):
                    torch.cuda.manual_seed(seed)
        yield
    finally:
        restore_rng_state(snapshot)


def rng_state_to_serialisable(snapshot: RngSnapshot) -> dict[str, Any]:
    """Split a snapshot into CPU tensors (payload file) and JSON-safe metadata."""
    py_version, py_keys, py_gauss = snapshot.python_state
    np_name, np_keys, np_pos, np_has_gauss, np_gauss = snapshot.numpy_state
    tensors: dict[str, torch.Tensor] = {
        "torch_cpu": snapshot.torch_cpu_state.to(torch.uint8).cpu(),
        "python_keys": torch.tensor(list(py_keys), dtype=torch.int64),
        "numpy_keys": torch.from_numpy(np.asarray(np_keys, dtype=np.int64).copy()),
    }
    for i, state in enumerate(snapshot.torch_cuda_states or []):
        tensors[f"torch_cuda_{i}"] = state.to(torch.uint8).cpu()
    meta = {
        "python_version": int(py_version),
        "python_gauss": py_gauss,
        "numpy_name": str(np_name),
        "numpy_pos": int(np_pos),
        "numpy_has_gauss": int(np_has_gauss),
        "numpy_gauss": float(np_gauss),
        "num_cuda_states": len(snapshot.torch_cuda_states or []),
    }
    return {"tensors": tensors, "meta": meta}


def rng_state_from_serialisable(payload: dict[str, Any]) -> RngSnapshot:
    tensors, meta = payload["tensors"], payload["meta"]
    py_state = (meta["python_version"], tuple(int(v) for v in tensors["python_keys"].tolist()), meta["python_gauss"])
    np_state = (meta["numpy_name"], np.asarray(tensors["numpy_keys"].tolist(), dtype=np.uint32), meta["numpy_pos"],
                meta["numpy_has_gauss"], meta["numpy_gauss"])
    count = int(meta.get("num_cuda_states", 0))
    cuda = [tensors[f"torch_cuda_{i}"] for i in range(count)] if count else None
    return RngSnapshot(py_state, np_state, tensors["torch_cpu"], cuda)
