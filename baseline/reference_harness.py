"""Reference arm of ``bench.py``: the unmodified reference, driven through its public API.

Imports only the reference package installed in ``baseline/_ref`` (its import
name is also ``hybrid_training``; ``bench.py`` removes this repository from
``sys.path`` before importing this module).  The step is the reference
engine's ``train_step`` (``src/hybrid_training/training/engine.py:352-422``)
spelled out, with the one addition the benchmark config asks for and the
reference engine lacks: the forward pass and loss run under
``torch.autocast(bfloat16)`` (fp32 master weights, as the reference keeps
them).  Model: ``TinyTransformer`` built by ``build_parallel_model`` (GPT-2-124M
shape, tied embeddings), wrapped in the reference's DDP (25 MB buckets);
optimizer: the reference's ``ShardedOptimizer`` (``torch.optim.AdamW``);
loss: the reference's ``cross_entropy_loss`` on full logits; gradient
scaler and metric reduction as in its engine.  Data: uniform random token
ids in pinned host memory.
"""

from __future__ import annotations

import os
from collections.abc import Callable

import torch
import torch.distributed as dist

from hybrid_training.config import (  # the reference package
    DDPConfig,
    ExperimentConfig,
    ModelConfig,
    OptimizerConfig,
    TopologyConfig,
    TrainingConfig,
)
from hybrid_training.distributed.context import init_distributed
from hybrid_training.optim.grad_scaler import GradScaler
from hybrid_training.optim.sharded_optimizer import ShardedOptimizer
from hybrid_training.parallel.hybrid import build_parallel_model
from hybrid_training.training.engine import cross_entropy_loss
from hybrid_training.utils.reproducibility import seed_everything

VOCAB = 50257


def _max_over_ranks(ms: float) -> float:
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _timed(fn: Callable[[], None]) -> float:
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    fn()
    b.record()
    torch.cuda.synchronize()
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
    return _max_over_ranks(a.elapsed_time(b))


def run(*, steps: int, warmup: int, micro_batch: int, seq: int, use_graph: bool = False,
        clock_start: Callable[[], None] | None = None, clock_stop: Callable[[], dict] | None = None) -> dict:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    cfg = ExperimentConfig(
        name="reference-gpt2-124m-ddp", backend="nccl", device="cuda", timeout_seconds=600.0,
        topology=TopologyConfig(data_parallel_size=world),
        model=ModelConfig(kind="transformer", hidden_size=768, num_layers=12, num_heads=12, vocab_size=VOCAB,
                          max_sequence_length=seq, tie_word_embeddings=True, activation="gelu"),
        optimizer=OptimizerConfig(learning_rate=6e-4, weight_decay=0.1, betas=(0.9, 0.95)),
        training=TrainingConfig(deterministic=False),
        ddp=DDPConfig(bucket_cap_mb=25.0),
    )
    ctx = init_distributed(cfg)
    seed_everything(cfg.training.seed, stream="model-init", deterministic=False)
    model = build_parallel_model(cfg, ctx)
    seed_everything(cfg.training.seed, stream="runtime", index=ctx.group("dp_shard").local_rank, deterministic=False)
    optimizer = ShardedOptimizer(model.optimizer_parameters(), cfg.optimizer, norm_group=model.norm_group, device=ctx.device)
    scaler = GradScaler(cfg.mixed_precision.scaler, ctx.group("world"), ctx.device)
    device = ctx.device
    gen = torch.Generator().manual_seed(1234 + ctx.rank)

    def host_batch() -> tuple[torch.Tensor, torch.Tensor]:
        tokens = torch.randint(0, VOCAB, (micro_batch, seq + 1), generator=gen)
        return tokens[:, :-1].contiguous().pin_memory(), tokens[:, 1:].contiguous().pin_memory()

    def step(x: torch.Tensor, y: torch.Tensor) -> float:
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = model(x)
            loss = cross_entropy_loss(logits, y)
        scaler.scale(loss).backward()
        local = float(loss.detach().item())
        model.finish_backward()
        params = model.optimizer_parameters()
        scaler.unscale_(params)
        scaler.step(optimizer, params, already_unscaled=True)
        scaler.update()
        optimizer.zero_grad(set_to_none=True)
        return model.reduce_metric(local)

    for _ in range(warmup):
        x, y = host_batch()
        step(x.to(device, non_blocking=True), y.to(device, non_blocking=True))
    dev_batches = [tuple(t.to(device) for t in host_batch()) for _ in range(steps)]
    host_batches = [host_batch() for _ in range(steps)]
    torch.cuda.synchronize()

    def device_loop() -> None:
        for x, y in dev_batches:
            step(x, y)

    if clock_start is not None:
        clock_start()
    device_ms = _timed(device_loop)
    clocks = clock_stop() if clock_stop is not None else {}
    losses: list[float] = []

    def e2e_loop() -> None:
        for x, y in host_batches:
            losses.append(step(x.to(device, non_blocking=True), y.to(device, non_blocking=True)))

    e2e_ms = _timed(e2e_loop)
    h2d = 2 * micro_batch * seq * 8
    if model.ddp is not None:
        model.ddp.teardown()
    ctx.shutdown()
    return {"device_ms": device_ms, "e2e_ms": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 8,
            "clocks": clocks, "loss": losses[-1] if losses else None}
