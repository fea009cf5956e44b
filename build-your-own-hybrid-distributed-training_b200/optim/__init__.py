"""Optimizers: fused flat AdamW, the sharded optimizer wrapper, loss scaling."""

from .fused_adamw import FusedAdamW
from .grad_scaler import GradScaler, GradScalerState
from .sharded_optimizer import (
    NormContribution,
    ShardedOptimizer,
    build_gradient_norm_contributions,
    build_inner_optimizer,
    distributed_gradient_norm,
)

__all__ = [
    "FusedAdamW",
    "GradScaler",
    "GradScalerState",
    "NormContribution",
    "ShardedOptimizer",
    "build_gradient_norm_contributions",
    "build_inner_optimizer",
    "distributed_gradient_norm",
]
