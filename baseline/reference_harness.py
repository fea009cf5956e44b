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

The Llama-shaped benchmark configurations have no exact counterpart in the
reference (it has no RMSNorm, RoPE, SwiGLU, GQA or vocabulary-parallel loss).
For them this arm runs the reference's own ``TinyTransformer`` at the same
width, depth, head count, feed-forward width, vocabulary and sequence length
(LayerNorm, learned positions, GELU feed-forward, multi-head attention with
materialised scores, full-logit output head), through the same stock
``build_parallel_model`` path, with the configuration's parallelism: FSDP
full shard with one unit per block (``llama_fsdp``), tensor + sequence
parallelism over all ranks (``llama_tp_sp``), or DP2 x TP(N/2) + SP with
gradient accumulation under ``no_sync`` (``llama_hybrid``).  ``shape`` in the
result records these differences.
"""

from __future__ import annotations

import contextlib
import os
from collections.abc import Callable

import torch
import torch.distributed as dist

from hybrid_training.config import (  # the reference package
    DDPConfig,
    ExperimentConfig,
    FSDPConfig,
    MixedPrecisionConfig,
    ModelConfig,
    OptimizerConfig,
    TensorParallelConfig,
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

# Llama-shaped tiers: (hidden, layers, heads, ffn, vocab) of the native configuration of the same name.
LLAMA_SHAPES = {
    "llama_fsdp": (2048, 24, 16, 5504, 32000),
    "llama_tp_sp": (4096, 32, 32, 14336, 128256),
    "llama_hybrid": (4096, 32, 32, 14336, 128256),
}


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


def _experiment(config: str, world: int, seq: int) -> tuple[ExperimentConfig, int]:
    """(reference ExperimentConfig, gradient accumulation) of one benchmark configuration."""
    if config == "gpt2_ddp":
        return ExperimentConfig(
            name="reference-gpt2-124m-ddp", backend="nccl", device="cuda", timeout_seconds=600.0,
            topology=TopologyConfig(data_parallel_size=world),
            model=ModelConfig(kind="transformer", hidden_size=768, num_layers=12, num_heads=12, vocab_size=VOCAB,
                              max_sequence_length=seq, tie_word_embeddings=True, activation="gelu"),
            optimizer=OptimizerConfig(learning_rate=6e-4, weight_decay=0.1, betas=(0.9, 0.95)),
            training=TrainingConfig(deterministic=False),
            ddp=DDPConfig(bucket_cap_mb=25.0),
        ), 1
    d, layers, heads, ffn, vocab = LLAMA_SHAPES[config]
    model = ModelConfig(kind="transformer", hidden_size=d, num_layers=layers, num_heads=heads, ffn_hidden_size=ffn,
                        vocab_size=vocab, max_sequence_length=seq, tie_word_embeddings=False, activation="gelu")
    common = dict(backend="nccl", device="cuda", timeout_seconds=900.0, model=model,
                  optimizer=OptimizerConfig(learning_rate=3e-4, weight_decay=0.1),
                  training=TrainingConfig(deterministic=False))
    if config == "llama_fsdp":
        # One FSDP unit per decoder block: the threshold lies above the largest sub-module of a
        # block (its feed-forward pair) and below the block itself.
        ffn_params = 2 * d * ffn + ffn + d
        return ExperimentConfig(name="reference-llama-1b3-fsdp", topology=TopologyConfig(shard_parallel_size=world),
                                fsdp=FSDPConfig(auto_wrap_min_num_params=ffn_params + 1),
                                mixed_precision=MixedPrecisionConfig(enabled=True, param_dtype="bfloat16"), **common), 1
    if config == "llama_tp_sp":
        return ExperimentConfig(name="reference-llama3-8b-tp-sp",
                                topology=TopologyConfig(tensor_parallel_size=world,
                                                        sequence_parallel_mode="tensor_group" if world > 1 else "disabled"),
                                tensor_parallel=TensorParallelConfig(sequence_parallel=world > 1), **common), 1
    tp = max(1, world // 2)
    return ExperimentConfig(name="reference-llama3-8b-hybrid",
                            topology=TopologyConfig(data_parallel_size=world // tp, tensor_parallel_size=tp,
                                                    sequence_parallel_mode="tensor_group" if tp > 1 else "disabled"),
                            tensor_parallel=TensorParallelConfig(sequence_parallel=tp > 1),
                            ddp=DDPConfig(bucket_cap_mb=25.0), **common), 4


def run(*, steps: int, warmup: int, micro_batch: int, seq: int, use_graph: bool = False,
        clock_start: Callable[[], None] | None = None, clock_stop: Callable[[], dict] | None = None,
        config: str = "gpt2_ddp", grad_accum: int = 1) -> dict:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    cfg, accum = _experiment(config, world, seq)
    vocab = cfg.model.vocab_size
    ctx = init_distributed(cfg)
    seed_everything(cfg.training.seed, stream="model-init", deterministic=False)
    model = build_parallel_model(cfg, ctx)
    seed_everything(cfg.training.seed, stream="runtime", index=ctx.group("dp_shard").local_rank, deterministic=False)
    optimizer = ShardedOptimizer(model.optimizer_parameters(), cfg.optimizer, norm_group=model.norm_group, device=ctx.device)
    scaler = GradScaler(cfg.mixed_precision.scaler, ctx.group("world"), ctx.device)
    device = ctx.device

    tp_rank_group = ctx.group("dp_shard")  # tensor/sequence peers must see the same tokens
    gen = torch.Generator().manual_seed(1234 + tp_rank_group.local_rank)

    def host_batch() -> list[tuple[torch.Tensor, torch.Tensor]]:
        out = []
        for _ in range(accum):
            tokens = torch.randint(0, vocab, (micro_batch, seq + 1), generator=gen)
            out.append((tokens[:, :-1].contiguous().pin_memory(), tokens[:, 1:].contiguous().pin_memory()))
        return out

    def step(micro: list[tuple[torch.Tensor, torch.Tensor]]) -> float:
        # The reference engine's train_step: no_sync on all but the last micro-batch, one host
        # read of the loss per micro-batch, then finish_backward / unscale / step / update.
        local = 0.0
        for i, (x, y) in enumerate(micro):
            ctxm = model.no_sync() if i < len(micro) - 1 else contextlib.nullcontext()
            with ctxm:
                with torch.autocast("cuda", dtype=torch.bfloat16):
                    logits = model(x)
                    loss = cross_entropy_loss(logits, y) / len(micro)
                scaler.scale(loss).backward()
            local += float(loss.detach().item())
        model.finish_backward()
        params = model.optimizer_parameters()
        scaler.unscale_(params)
        scaler.step(optimizer, params, already_unscaled=True)
        scaler.update()
        optimizer.zero_grad(set_to_none=True)
        return model.reduce_metric(local)

    def to_device(micro: list[tuple[torch.Tensor, torch.Tensor]]) -> list[tuple[torch.Tensor, torch.Tensor]]:
        return [(x.to(device, non_blocking=True), y.to(device, non_blocking=True)) for x, y in micro]

    for _ in range(warmup):
        step(to_device(host_batch()))
    dev_batches = [to_device(host_batch()) for _ in range(steps)]
    host_batches = [host_batch() for _ in range(steps)]
    torch.cuda.synchronize()

    def device_loop() -> None:
        for micro in dev_batches:
            step(micro)

    if clock_start is not None:
        clock_start()
    device_ms = _timed(device_loop)
    clocks = clock_stop() if clock_stop is not None else {}
    losses: list[float] = []

    def e2e_loop() -> None:
        for micro in host_batches:
            losses.append(step(to_device(micro)))

    e2e_ms = _timed(e2e_loop)
    h2d = 2 * micro_batch * seq * 8 * accum
    peak = torch.cuda.max_memory_allocated(device)
    replicas = cfg.topology.data_parallel_size * cfg.topology.shard_parallel_size
    if model.ddp is not None:
        model.ddp.teardown()
    ctx.shutdown()
    shape = None
    if config != "gpt2_ddp":
        d, layers, heads, ffn, v = LLAMA_SHAPES[config]
        shape = (f"reference TinyTransformer d{d} L{layers} {heads} heads (MHA) GELU ffn {ffn} V{v}, LayerNorm, learned "
                 "positions, materialised attention scores, full-logit head")
    return {"device_ms": device_ms, "e2e_ms": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 8 * accum,
            "clocks": clocks, "loss": losses[-1] if losses else None, "peak_memory_bytes": peak,
            "tokens_per_step": micro_batch * seq * accum * replicas, "shape": shape}
