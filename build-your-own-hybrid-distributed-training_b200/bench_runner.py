"""Runner behind ``bench.py --impl native``: the GPT-2-124M DDP step through the public engine API.

``run`` builds the experiment with :class:`TrainingEngine` (one process per GPU,
NCCL process groups, DDP over the data-parallel group with the in-kernel
bucket all-reduce, bf16 compute with fp32 master weights, fused AdamW, CUDA
graph step) and returns device-timed and end-to-end step times (max over
ranks), the bytes crossing the host/device boundary per step, and the number
of native kernel launches per timed region.
"""

from __future__ import annotations

import os
from collections.abc import Callable
from typing import Any

import torch
import torch.distributed as dist

from .config import (
    DataConfig,
    DDPConfig,
    FSDPConfig,
    ExperimentConfig,
    MixedPrecisionConfig,
    ModelConfig,
    OptimizerConfig,
    TensorParallelConfig,
    TopologyConfig,
    TrainingConfig,
)
from .distributed.collectives import observe_collectives
from .distributed.context import init_distributed
from .training.data import Batch
from .training.engine import TrainingEngine

__all__ = ["count_native_launches", "run"]


def count_native_launches(fn: Callable[[], Any]) -> int:
    """Number of kernels from this package's native module launched by ``fn()`` (profiled, untimed)."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return sum(1 for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA and "ht::" in e.name)


def _max_over_ranks(ms: float) -> float:
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=dist.group.WORLD)
    return float(t.item())


def _timed(fn: Callable[[], None]) -> float:
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier(group=dist.group.WORLD)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    fn()
    stop.record()
    torch.cuda.synchronize()
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier(group=dist.group.WORLD)
    return _max_over_ranks(start.elapsed_time(stop))


# Benchmark configurations: name -> (description, parallelism, builder).
CONFIGS = ("gpt2_ddp", "llama_fsdp", "llama_tp_sp", "llama_hybrid")


def experiment(world: int, *, micro_batch: int, seq: int, samples: int, use_graph: bool, config: str = "gpt2_ddp",
               grad_accum: int = 1, overlap_step: bool = False) -> ExperimentConfig:
    """The ExperimentConfig of one benchmark configuration on ``world`` GPUs."""
    common = dict(backend="nccl", device="cuda", timeout_seconds=600.0,
                  data=DataConfig(micro_batch_size=micro_batch, sequence_length=seq, num_train_samples=samples,
                                  num_eval_samples=0, token_distribution="uniform", shuffle=False),
                  mixed_precision=MixedPrecisionConfig(enabled=True, param_dtype="bfloat16"))
    # CUDA-graph replay is used for the data-parallel step; the sharded / tensor-parallel
    # configurations run eagerly.
    training = TrainingConfig(max_steps=1_000_000, log_every_steps=0, deterministic=False,
                              cuda_graph=use_graph and config == "gpt2_ddp", gradient_accumulation_steps=grad_accum,
                              overlap_optimizer_step=overlap_step)
    if config == "gpt2_ddp":
        return ExperimentConfig(name="bench-gpt2-124m-ddp", topology=TopologyConfig(data_parallel_size=world),
                                model=ModelConfig.gpt2_124m(),
                                optimizer=OptimizerConfig(learning_rate=6e-4, weight_decay=0.1, betas=(0.9, 0.95)),
                                training=training, ddp=DDPConfig(bucket_cap_mb=25.0), **common)
    if config == "llama_fsdp":  # full shard, one flat parameter per decoder block
        return ExperimentConfig(name="bench-llama-1b3-fsdp", topology=TopologyConfig(shard_parallel_size=world),
                                model=ModelConfig.llama_1b3(), optimizer=OptimizerConfig(learning_rate=3e-4, weight_decay=0.1),
                                training=training, fsdp=FSDPConfig(auto_wrap_min_num_params=10_000_000), **common)
    if config == "llama_tp_sp":  # tensor + sequence parallel over every GPU
        return ExperimentConfig(name="bench-llama3-8b-tp-sp",
                                topology=TopologyConfig(tensor_parallel_size=world,
                                                        sequence_parallel_mode="tensor_group" if world > 1 else "disabled"),
                                tensor_parallel=TensorParallelConfig(sequence_parallel=world > 1),
                                model=ModelConfig.llama3_8b(), optimizer=OptimizerConfig(learning_rate=3e-4, weight_decay=0.1),
                                training=training, **common)
    if config == "llama_hybrid":  # DP2 x TP(world/2) with SP
        tp = max(1, world // 2)
        return ExperimentConfig(name="bench-llama3-8b-hybrid",
                                topology=TopologyConfig(data_parallel_size=world // tp, tensor_parallel_size=tp,
                                                        sequence_parallel_mode="tensor_group" if tp > 1 else "disabled"),
                                tensor_parallel=TensorParallelConfig(sequence_parallel=tp > 1),
                                model=ModelConfig.llama3_8b(), optimizer=OptimizerConfig(learning_rate=3e-4, weight_decay=0.1),
                                training=training, ddp=DDPConfig(bucket_cap_mb=25.0), **common)
    raise ValueError(f"unknown benchmark config {config!r}; expected one of {CONFIGS}")


def _exposed_communication_ms(engine: TrainingEngine, stream: Any, take: Callable[[], list[Batch]], steps: int,
                               grad_accum: int, cfg: ExperimentConfig) -> float | None:
    """Per-step time that gradient communication adds to the data-parallel step.

    Both loops run eagerly: the same steps with and without the gradient reduction
    (``no_sync``); the difference is the communication the backward pass did not hide.
    Only defined for data-parallel (DDP) configurations.
    """
    if cfg.topology.data_parallel_size <= 1 or cfg.topology.shard_parallel_size > 1 or cfg.topology.tensor_parallel_size > 1:
        return None
    dev = engine.context.device
    engine.graph_enabled = False
    batches = [[mb.to(dev) for mb in take()] for _ in range(2 * steps + 2)]
    for b in batches[:2]:
        engine.train_step(iter(b), read_metrics=False)

    def synced() -> None:
        for b in batches[2:2 + steps]:
            engine.train_step(iter(b), read_metrics=False)

    def local() -> None:
        with engine.model.no_sync():
            for b in batches[2 + steps:]:
                engine.train_step(iter(b), read_metrics=False)

    full = _timed(synced)
    compute = _timed(local)
    engine.graph_enabled = True
    return max(0.0, (full - compute) / steps)


def run(*, steps: int, warmup: int, micro_batch: int, seq: int, use_graph: bool = True,
        clock_start: Callable[[], None] | None = None, clock_stop: Callable[[], dict] | None = None,
        config: str = "gpt2_ddp", grad_accum: int = 1, overlap_step: bool = False) -> dict:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    cfg = experiment(world, micro_batch=micro_batch, seq=seq,
                     samples=micro_batch * world * grad_accum * (2 * steps + warmup + 9), use_graph=use_graph,
                     config=config, grad_accum=grad_accum, overlap_step=overlap_step)
    ctx = init_distributed(cfg)
    engine = TrainingEngine(cfg, ctx)
    stream = engine.batch_stream(host=True)
    dev = ctx.device

    def step(batch: list[Batch], read: bool) -> Any:
        return engine.train_step(iter(batch), read_metrics=read)

    launches_per_step = 0
    def take() -> list[Batch]:
        return [next(stream) for _ in range(grad_accum)]

    comm: dict[str, dict[str, float]] = {}
    for i in range(warmup):
        b = take()
        if i == 0 and ctx.rank == 0 and os.environ.get("HT_COUNT_LAUNCHES", "1") != "0":
            launches_per_step = count_native_launches(lambda: step(b, True))
        else:
            step(b, True)
    # One more untimed step, run eagerly with every collective counted (a replayed graph issues
    # the same collectives without passing through Python).
    graph = engine.graph_enabled
    engine.graph_enabled = False
    with observe_collectives() as rec:
        step(take(), True)
    engine.graph_enabled = graph
    comm = {k: {"calls": v.calls, "bytes": v.bytes} for k, v in sorted(rec.by_operation.items())}
    # device-resident batches for the device-timed loop
    dev_batches = [[mb.to(dev) for mb in take()] for _ in range(steps)]
    host_batches = [take() for _ in range(steps)]
    torch.cuda.synchronize()

    def device_loop() -> None:
        for b in dev_batches:
            step(b, False)

    if clock_start is not None:
        clock_start()
    device_ms = _timed(device_loop)
    clocks = clock_stop() if clock_stop is not None else {}
    losses: list[float] = []

    def e2e_loop() -> None:
        for b in host_batches:
            losses.append(step(b, True).loss)

    e2e_ms = _timed(e2e_loop)
    exposed = _exposed_communication_ms(engine, stream, take, steps, grad_accum, cfg) if world > 1 else 0.0
    h2d = sum(mb.inputs.numel() * mb.inputs.element_size() + mb.targets.numel() * mb.targets.element_size()
              for mb in host_batches[0])
    replicas = cfg.topology.data_parallel_size * cfg.topology.shard_parallel_size
    memory = _memory_record(engine, dev)
    engine.close()
    ctx.shutdown()
    return {"device_ms": device_ms, "e2e_ms": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
            "gpu_launches": launches_per_step * steps, "clocks": clocks, "loss": losses[-1] if losses else None,
            "exposed_comm_ms_per_step": exposed, "tokens_per_step": micro_batch * seq * grad_accum * replicas,
            "parallelism": cfg.topology.describe() if hasattr(cfg.topology, "describe") else None,
            "communication_per_step": comm, **memory}


def _memory_record(engine: TrainingEngine, device: torch.device) -> dict[str, int]:
    """Parameter, optimizer-state and peak device bytes of this rank (the benchmark sweep's memory columns)."""
    params = {id(p): p for p in engine.model.parameters()}
    inner = engine.optimizer.inner
    opt_bytes = 0
    for st in getattr(inner, "state", {}).values():
        for v in st.values():
            if torch.is_tensor(v):
                opt_bytes += v.numel() * v.element_size()
    flat = getattr(inner, "flat_parameters", None)
    master = flat.numel() * flat.element_size() if torch.is_tensor(flat) else 0
    return {"parameter_bytes": sum(p.numel() * p.element_size() for p in params.values()),
            "master_parameter_bytes": master, "optimizer_state_bytes": opt_bytes,
            "peak_memory_bytes": int(torch.cuda.max_memory_allocated(device))}
