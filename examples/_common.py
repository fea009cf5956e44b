"""Shared command line and reporting for the example programs (run them with torchrun)."""

from __future__ import annotations

import argparse
import dataclasses
import sys
from pathlib import Path
from collections.abc import Callable
from typing import Any

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from hybrid_training.config import ExperimentConfig, load_experiment_config  # noqa: E402
from hybrid_training.distributed.context import DistributedContext  # noqa: E402
from hybrid_training.distributed.launch import torchrun_environment_summary  # noqa: E402
from hybrid_training.logging import configure_logging  # noqa: E402

CONFIGS = ROOT / "configs"


def parser(description: str, default_config: str) -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=description, formatter_class=argparse.ArgumentDefaultsHelpFormatter)
    p.add_argument("--config", default=str(CONFIGS / default_config), help="YAML experiment configuration")
    p.add_argument("--steps", type=int, default=None, help="override training.max_steps")
    p.add_argument("--seed", type=int, default=None, help="override training.seed")
    p.add_argument("--backend", default=None, choices=["auto", "gloo", "nccl"])
    p.add_argument("--device", default=None, choices=["auto", "cpu", "cuda"])
    p.add_argument("--checkpoint-dir", default=None, help="override checkpoint.directory")
    p.add_argument("--log-level", default="INFO", choices=["DEBUG", "INFO", "WARNING", "ERROR"])
    p.add_argument("--show-topology", action="store_true", help="print this rank's coordinates and groups")
    return p


def load_config(args: argparse.Namespace) -> ExperimentConfig:
    configure_logging(args.log_level)
    cfg = load_experiment_config(args.config)
    if args.backend is not None:
        cfg = dataclasses.replace(cfg, backend=args.backend)
    if args.device is not None:
        cfg = dataclasses.replace(cfg, device=args.device)
    if args.steps is not None:
        cfg = dataclasses.replace(cfg, training=dataclasses.replace(cfg.training, max_steps=args.steps))
    if args.seed is not None:
        cfg = dataclasses.replace(cfg, training=dataclasses.replace(cfg.training, seed=args.seed))
    if args.checkpoint_dir is not None:
        cfg = dataclasses.replace(cfg, checkpoint=dataclasses.replace(cfg.checkpoint, directory=args.checkpoint_dir))
    return cfg


def report_environment(context: DistributedContext, *, show_topology: bool) -> None:
    if context.is_primary:
        print("launch environment:")
        for k, v in torchrun_environment_summary().items():
            print(f"  {k:<22} {v}")
    if show_topology:
        print(context.describe())


def report_result(context: DistributedContext, engine: Any) -> None:
    counts = engine.parameter_count()
    if not context.is_primary:
        return
    print("=" * 72)
    print(f"strategy            : {engine.model.description.strategy}")
    print(f"world size          : {context.world_size} ({context.backend} on {context.device})")
    print(f"parameters (local)  : {counts['local']:,}")
    print(f"parameters (global) : {counts['global']:,}")
    print(f"final state         : {engine.state.describe()}")
    if engine.history:
        print(f"loss                : {engine.history[0].loss:.6f} -> {engine.history[-1].loss:.6f}")
    m = engine.model.memory_summary()
    print(f"memory (per rank)   : shard={m['shard_bytes']:,}B grad={m['grad_shard_bytes']:,}B padding={m['padding_bytes']:,}B "
          f"units={m['units']}")
    print(engine.communication_summary())
    print("=" * 72)


Hook = Callable[[DistributedContext, Any], None]


def primary_print(context: DistributedContext, *lines: str) -> None:
    if context.is_primary:
        for line in lines:
            print(line)


def run_training(description: str, default_config: str, *, before: Hook | None = None, after: Hook | None = None) -> None:
    """Build the engine for ``--config``, run it, report.

    ``before`` runs on every rank once the model is wrapped (before the first step) and ``after``
    once training has finished; the example programs use them to show what their strategy does.
    Both may call collectives: every rank runs them.
    """
    from hybrid_training.distributed import distributed_context
    from hybrid_training.training import TrainingEngine

    args = parser(description, default_config).parse_args()
    cfg = load_config(args)
    with distributed_context(cfg) as ctx:
        report_environment(ctx, show_topology=args.show_topology)
        engine = TrainingEngine(cfg, ctx)
        if ctx.is_primary:
            print(engine.model.description.render())
        if before is not None:
            before(ctx, engine)
        engine.train()
        if after is not None:
            after(ctx, engine)
        report_result(ctx, engine)
        engine.close()
