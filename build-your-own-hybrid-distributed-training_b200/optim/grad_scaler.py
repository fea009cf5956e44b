"""Dynamic loss scaling for fp16 with a world-wide overflow vote.

Behaviour of ``src/hybrid_training/optim/grad_scaler.py:52-298``: ``scale``
multiplies the loss; ``unscale_`` divides gradients and detects non-finite
values, with a MAX all-reduce so every rank skips the same step; ``update``
backs off on overflow and grows after ``growth_interval`` clean steps.
bf16 does not need (and the config rejects) loss scaling; with the scaler
disabled the training engine skips the overflow vote entirely, which removes
a host synchronisation from every step.
"""

from __future__ import annotations

from collections.abc import Iterable, Sequence
from dataclasses import dataclass
from typing import Any

import torch
import torch.nn as nn

from ..config import GradScalerConfig
from ..distributed.collectives import CommunicationRecorder, ReduceOp, all_reduce
from ..distributed.groups import GroupHandle
from ..logging import get_logger

__all__ = ["GradScaler", "GradScalerState"]

_LOG = get_logger(__name__)


@dataclass
class GradScalerState:
    scale: float
    growth_tracker: int = 0
    total_steps: int = 0
    skipped_steps: int = 0

    def as_dict(self) -> dict[str, float]:
        return {"scale": float(self.scale), "growth_tracker": int(self.growth_tracker), "total_steps": int(self.total_steps),
                "skipped_steps": int(self.skipped_steps)}

    @classmethod
    def from_dict(cls, payload: dict[str, Any]) -> GradScalerState:
        return cls(float(payload["scale"]), int(payload.get("growth_tracker", 0)), int(payload.get("total_steps", 0)),
                   int(payload.get("skipped_steps", 0)))


def _grad(p: nn.Parameter) -> torch.Tensor | None:
    if p.grad is not None:
        return p.grad
    mg = getattr(p, "main_grad", None)
    return None if mg is None or getattr(p, "main_grad_fresh", True) else mg


class GradScaler:
    def __init__(self, config: GradScalerConfig, group: GroupHandle, device: torch.device, *,
                 recorder: CommunicationRecorder | None = None) -> None:
        self._config, self._group, self._device, self._recorder = config, group, device, recorder
        self._state = GradScalerState(scale=config.init_scale if config.enabled else 1.0)
        self._unscaled = False
        self._skipped_last = False

    enabled = property(lambda self: self._config.enabled)
    state = property(lambda self: self._state)

    @property
    def scale_value(self) -> float:
        return self._state.scale if self._config.enabled else 1.0

    def scale(self, loss: torch.Tensor) -> torch.Tensor:
        if not self._config.enabled:
            return loss
        self._unscaled = False
        return loss * self._state.scale

    def unscale_(self, parameters: Iterable[nn.Parameter]) -> bool:
        grads = [g for g in (_grad(p) for p in parameters) if g is not None]
        if self._config.enabled:
            inv = 1.0 / self._state.scale
            for g in grads:
                g.detach().mul_(inv)
            self._unscaled = True
        return self._vote(grads)

    def _vote(self, grads: Sequence[torch.Tensor]) -> bool:
        """MAX-reduce a local non-finite flag so all ranks agree to skip."""
        flag = torch.zeros(1, dtype=torch.float32, device=self._device)
        if grads:
            bad = torch.stack([(~torch.isfinite(g.detach())).any() for g in grads]).any()
            flag.copy_(bad.float().reshape(1).to(self._device))
        all_reduce(flag, self._group, op=ReduceOp.MAX, recorder=self._recorder).wait()
        return bool(flag.item() > 0)

    def _detect_non_finite(self, parameters: Sequence[nn.Parameter]) -> bool:
        return self._vote([g for g in (_grad(p) for p in parameters) if g is not None])

    def step(self, optimizer: Any, parameters: Iterable[nn.Parameter], *, already_unscaled: bool = False) -> bool:
        params = list(parameters)
        bad = self._detect_non_finite(params) if (already_unscaled or self._unscaled) else self.unscale_(params)
        self._state.total_steps += 1
        self._skipped_last = bad
        if bad:
            self._state.skipped_steps += 1
            _LOG.warning("non-finite gradient on at least one rank; skipping step %d, loss scale %.1f", self._state.total_steps,
                         self._state.scale)
            return False
        optimizer.step()
        return True

    def update(self, *, found_non_finite: bool | None = None) -> float:
        if not self._config.enabled:
            return 1.0
        overflow = self._skipped_last if found_non_finite is None else found_non_finite
        if overflow:
            self._state.scale = max(self._state.scale * self._config.backoff_factor, 1.0)
            self._state.growth_tracker = 0
        else:
            self._state.growth_tracker += 1
            if self._state.growth_tracker >= self._config.growth_interval:
                self._state.scale = min(self._state.scale * self._config.growth_factor, self._config.max_scale)
                self._state.growth_tracker = 0
        self._unscaled = False
        return self._state.scale

    @property
    def last_step_skipped(self) -> bool:
        return self._skipped_last

    def state_dict(self) -> dict[str, float]:
        return self._state.as_dict()

    def load_state_dict(self, payload: dict[str, Any]) -> None:
        self._state = GradScalerState.from_dict(payload)
        self._unscaled = False

    def __repr__(self) -> str:
        return f"GradScaler(enabled={self._config.enabled}, scale={self.scale_value}, skipped={self._state.skipped_steps}/{self._state.total_steps})"
