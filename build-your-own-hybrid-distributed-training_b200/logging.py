"""Rank-aware logging.

Records are tagged with ``rank R/W`` and the 4-D grid coordinates of the
emitting rank; ``primary_only`` records are dropped on every rank but 0; and
``HYBRID_LOG_FORMAT=json`` switches to one JSON object per line.  Same
behaviour as the reference (``src/hybrid_training/logging.py:46-285``).
"""

from __future__ import annotations

import json
import logging
import os
import sys
import time
from collections.abc import Iterator
from contextlib import contextmanager
from dataclasses import dataclass
from typing import Any

__all__ = [
    "LogContext",
    "RankFilter",
    "configure_logging",
    "get_log_context",
    "get_logger",
    "log_context",
    "log_primary",
    "set_log_context",
]

_ROOT = "hybrid_training"
_TEXT_FORMAT = "%(asctime)s [%(rank_tag)s] %(levelname)s %(name)s | %(message)s"


@dataclass(frozen=True)
class LogContext:
    """Identity of the current process inside the job."""

    rank: int = -1
    world_size: int = 1
    local_rank: int = 0
    coordinates: str = ""

    @property
    def tag(self) -> str:
        base = "rank ?" if self.rank < 0 else f"rank {self.rank}/{self.world_size}"
        return f"{base} {self.coordinates}" if self.coordinates else base

    @property
    def is_primary(self) -> bool:
        return self.rank <= 0


_CURRENT = LogContext()


def set_log_context(context: LogContext) -> LogContext:
    """Install ``context`` for every subsequent record; returns the previous one."""
    global _CURRENT
    previous, _CURRENT = _CURRENT, context
    return previous


def get_log_context() -> LogContext:
    return _CURRENT


@contextmanager
def log_context(context: LogContext) -> Iterator[LogContext]:
    previous = set_log_context(context)
    try:
        yield context
    finally:
        set_log_context(previous)


class RankFilter(logging.Filter):
    """Stamps rank fields on every record and drops non-primary ``primary_only`` records."""

    def filter(self, record: logging.LogRecord) -> bool:
        ctx = _CURRENT
        record.rank = ctx.rank
        record.world_size = ctx.world_size
        record.local_rank = ctx.local_rank
        record.coordinates = ctx.coordinates
        record.rank_tag = ctx.tag
        return ctx.is_primary or not getattr(record, "primary_only", False)


_RESERVED = frozenset(
    logging.LogRecord("", 0, "", 0, "", (), None).__dict__.keys()
    | {"message", "asctime", "rank", "world_size", "local_rank", "coordinates", "rank_tag", "primary_only", "taskName"}
)


def _plain(value: Any) -> Any:
    if isinstance(value, (str, int, float, bool)) or value is None:
        return value
    if isinstance(value, (list, tuple)):
        return [_plain(v) for v in value]
    if isinstance(value, dict):
        return {str(k): _plain(v) for k, v in value.items()}
    return repr(value)


class JsonFormatter(logging.Formatter):
    """One JSON object per record, with any ``extra=`` fields under ``extra``."""

    def format(self, record: logging.LogRecord) -> str:
        out: dict[str, Any] = {
            "time": time.strftime("%Y-%m-%dT%H:%M:%S", time.localtime(record.created)),
            "level": record.levelname,
            "logger": record.name,
            "rank": getattr(record, "rank", -1),
            "world_size": getattr(record, "world_size", 1),
            "local_rank": getattr(record, "local_rank", 0),
            "coordinates": getattr(record, "coordinates", ""),
            "message": record.getMessage(),
        }
        extra = {k: _plain(v) for k, v in record.__dict__.items() if k not in _RESERVED and not k.startswith("_")}
        if extra:
            out["extra"] = extra
        if record.exc_info:
            out["exception"] = self.formatException(record.exc_info)
        return json.dumps(out, sort_keys=True)


def configure_logging(
    level: int | str = logging.INFO, *, fmt: str | None = None, stream: Any = None, force: bool = False
) -> logging.Logger:
    """Attach one rank-aware handler to the package's root logger."""
    style = (fmt or os.environ.get("HYBRID_LOG_FORMAT") or "text").lower()
    if style not in ("text", "json"):
        raise ValueError(f"log format is 'text' or 'json', not {style!r}")
    logger = logging.getLogger(_ROOT)
    if logger.handlers and not force:
        logger.setLevel(level)
        return logger
    for handler in list(logger.handlers):
        logger.removeHandler(handler)
    handler = logging.StreamHandler(stream if stream is not None else sys.stderr)
    handler.setFormatter(JsonFormatter() if style == "json" else logging.Formatter(_TEXT_FORMAT))
    handler.addFilter(RankFilter())
    logger.addHandler(handler)
    logger.setLevel(level)
    logger.propagate = False
    return logger


def get_logger(name: str) -> logging.Logger:
    """Return a logger below the package root (``hybrid_training.<name>``)."""
    if name == _ROOT or name.startswith(_ROOT + "."):
        return logging.getLogger(name)
    return logging.getLogger(f"{_ROOT}.{name}")


def log_primary(logger: logging.Logger, level: int, message: str, **extra: Any) -> None:
    """Log only on the primary rank."""
    logger.log(level, message, extra={"primary_only": True, **extra})
