"""Multi-layer perceptron (the FSDP/DDP correctness model).

``[Linear -> activation] x L -> Linear`` with seeded initialisation, and the
tensor-parallel variant built from :class:`TensorParallelMLPBlock`; same
structure and parameter names as ``src/hybrid_training/models/mlp.py:45-226``
so gradients can be compared against a single-process run.  GELU is the tanh
approximation.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import ModelConfig
from ..distributed.groups import GroupHandle
from ..errors import ConfigurationError, format_error
from ..utils.reproducibility import derive_seed, temporary_seed

__all__ = ["MLP", "MLPBlock", "build_activation"]


def build_activation(name: str) -> Callable[[torch.Tensor], torch.Tensor]:
    if name == "gelu":
        return lambda x: F.gelu(x, approximate="tanh")
    if name == "relu":
        return F.relu
    if name == "swiglu":
        from .. import ops

        return ops.swiglu
    raise ConfigurationError(format_error("models.build_activation", "unknown activation", expected=["gelu", "relu", "swiglu"],
                                          observed=name, resolution="use 'gelu', 'relu' or 'swiglu'"))


class MLPBlock(nn.Module):
    def __init__(self, in_features: int, out_features: int, *, activation: str = "gelu", bias: bool = True) -> None:
        super().__init__()
        self.linear = nn.Linear(in_features, out_features, bias=bias)
        self.activation_name = activation
        self._activation = build_activation(activation)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._activation(self.linear(x))


class MLP(nn.Module):
    """``blocks`` (width ``hidden_size``) followed by a ``head`` to ``output_size``."""

    def __init__(self, config: ModelConfig, *, seed: int = 0, bias: bool = True, tensor_parallel_group: GroupHandle | None = None,
                 device: torch.device | None = None, dtype: torch.dtype | None = None) -> None:
        super().__init__()
        self.config = config
        self.tensor_parallel_group = tensor_parallel_group
        factory: dict[str, Any] = {k: v for k, v in (("device", device), ("dtype", dtype)) if v is not None}
        tp = tensor_parallel_group is not None and tensor_parallel_group.size > 1
        with temporary_seed(derive_seed(seed, "model-init")):
            widths = [config.input_size] + [config.hidden_size] * config.num_layers
            blocks: list[nn.Module] = []
            for i in range(config.num_layers):
                if tp:
                    from ..parallel.tensor_parallel import TensorParallelMLPBlock

                    blocks.append(TensorParallelMLPBlock(widths[i], widths[i + 1], tensor_parallel_group, activation=config.activation,
                                                         bias=bias, **factory))
                else:
                    blocks.append(MLPBlock(widths[i], widths[i + 1], activation=config.activation, bias=bias))
            self.blocks = nn.ModuleList(blocks)
            self.head = nn.Linear(config.hidden_size, config.output_size, bias=bias, **factory)
        if not tp and factory:
            self.to(**factory)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for block in self.blocks:
            x = block(x)
        return self.head(x)

    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters())

    def __repr__(self) -> str:
        tp = self.tensor_parallel_group.size if self.tensor_parallel_group is not None else 1
        c = self.config
        return f"MLP(in={c.input_size}, hidden={c.hidden_size}, layers={c.num_layers}, out={c.output_size}, tensor_parallel={tp})"
