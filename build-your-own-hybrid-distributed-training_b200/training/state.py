"""Training progress (JSON-only) and the pure-function learning-rate schedule.

Same fields and schedule shapes as ``src/hybrid_training/training/state.py:22-215``:
linear warm-up from ``lr/warmup`` to ``lr``, then constant, linear or cosine
decay to ``min_lr_ratio * lr`` at ``total_steps``.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field
from typing import Any

from ..config import SchedulerConfig
from ..errors import ConfigurationError, format_error

__all__ = ["LearningRateSchedule", "TrainingState"]


@dataclass
class TrainingState:
    step: int = 0
    epoch: int = 0
    micro_step: int = 0
    samples_seen: int = 0
    batches_in_epoch: int = 0
    last_loss: float = float("nan")
    best_eval_loss: float = float("inf")
    skipped_steps: int = 0

    def as_dict(self) -> dict[str, Any]:
        out = asdict(self)
        out["last_loss"] = None if math.isnan(self.last_loss) else self.last_loss
        out["best_eval_loss"] = None if math.isinf(self.best_eval_loss) else self.best_eval_loss
        return out

    @classmethod
    def from_dict(cls, payload: dict[str, Any]) -> TrainingState:
        data = dict(payload)
        if data.get("last_loss") is None:
            data["last_loss"] = float("nan")
        if data.get("best_eval_loss") is None:
            data["best_eval_loss"] = float("inf")
        return cls(**{k: v for k, v in data.items() if k in cls.__dataclass_fields__})

    def advance_step(self, *, samples: int) -> None:
        self.step += 1
        self.samples_seen += samples
        self.micro_step = 0

    def describe(self) -> str:
        loss = "nan" if math.isnan(self.last_loss) else f"{self.last_loss:.6f}"
        return f"step={self.step} epoch={self.epoch} samples={self.samples_seen} loss={loss} skipped={self.skipped_steps}"


@dataclass
class LearningRateSchedule:
    config: SchedulerConfig
    base_learning_rate: float
    total_steps: int = field(default=1)

    def __post_init__(self) -> None:
        if self.total_steps < 1:
            raise ConfigurationError(format_error("training.LearningRateSchedule", "the schedule needs one or more total steps", expected=">= 1",
                                                  observed=self.total_steps, resolution="use the run length (training.max_steps)"))
        if self.config.warmup_steps >= self.total_steps and self.config.name != "constant":
            raise ConfigurationError(format_error("training.LearningRateSchedule", "warm-up lasts the whole run, so decay never starts",
                                                  expected=f"warmup_steps < {self.total_steps}", observed=self.config.warmup_steps,
                                                  resolution="make warm-up shorter than the run"))

    def value_at(self, step: int) -> float:
        warm = self.config.warmup_steps
        if warm > 0 and step < warm:
            return self.base_learning_rate * (step + 1) / warm
        if self.config.name == "constant":
            return self.base_learning_rate
        progress = min(max((step - warm) / max(self.total_steps - warm, 1), 0.0), 1.0)
        floor = self.config.min_lr_ratio
        shape = (1.0 - progress) if self.config.name == "linear" else 0.5 * (1.0 + math.cos(math.pi * progress))
        return self.base_learning_rate * (floor + (1.0 - floor) * shape)

    def state_dict(self) -> dict[str, Any]:
        return {"name": self.config.name, "warmup_steps": self.config.warmup_steps, "min_lr_ratio": self.config.min_lr_ratio,
                "base_learning_rate": self.base_learning_rate, "total_steps": self.total_steps}

    @classmethod
    def from_state_dict(cls, payload: dict[str, Any]) -> LearningRateSchedule:
        cfg = SchedulerConfig(name=payload["name"], warmup_steps=int(payload["warmup_steps"]), min_lr_ratio=float(payload["min_lr_ratio"]))
        return cls(config=cfg, base_learning_rate=float(payload["base_learning_rate"]), total_steps=int(payload["total_steps"]))
