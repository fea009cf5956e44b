"""The training engine: one loop for every strategy.

Reference behaviour (``src/hybrid_training/training/engine.py:157-594``): build
the parallel model, the sharded optimizer, the LR schedule and the loss
scaler; per step run ``gradient_accumulation_steps`` micro-batches (all but
the last inside ``no_sync``), ``finish_backward``, unscale, clip, step, update,
zero; reduce the loss over ``dp_shard``; evaluate and checkpoint on schedule;
resume from a checkpoint (model, optimizer, RNG, schedule, data position).

B200-native changes:

* the step keeps the loss, the gradient norm and the clip coefficient on the
  device; the host reads the reduced loss once at the end of the step (the
  reference synchronises after every micro-batch and inside clipping and
  overflow detection);
* transformer losses come from the fused head + vocab-parallel cross-entropy
  (the model is called with ``targets``);
* with ``training.cuda_graph`` the whole steady-state step -- forward,
  backward, gradient reductions, clipping and the fused AdamW update -- is
  captured once in a CUDA graph and replayed; the only per-step host work is
  the pinned host-to-device copy of the batch, the learning-rate/step update
  of the optimizer's device vector and the loss readback.
"""

from __future__ import annotations

import time
from collections.abc import Callable
from dataclasses import dataclass, field, replace
from pathlib import Path
from typing import TYPE_CHECKING, Any

import torch
import torch.nn.functional as F

from ..config import ExperimentConfig
from ..distributed.collectives import CommunicationRecorder, ReduceOp, all_reduce, sum_scalar
from ..distributed.context import DistributedContext
from ..errors import ConfigurationError, format_error
from ..logging import get_logger
from ..optim.fused_adamw import FusedAdamW
from ..optim.overlapped_step import OverlappedAdamW
from ..optim.grad_scaler import GradScaler
from ..optim.sharded_optimizer import ShardedOptimizer
from ..parallel.hybrid import HybridModel, build_parallel_model
from ..utils.memory import MemorySnapshot, capture_memory, reset_peak_memory
from ..utils.reproducibility import seed_everything
from ..utils.tracing import trace_range
from .data import Batch, DistributedBatchSampler, SyntheticDataLoader, build_dataset
from .state import LearningRateSchedule, TrainingState

if TYPE_CHECKING:
    from ..checkpoint.reader import LoadedCheckpoint

__all__ = ["StepMetrics", "TrainingEngine", "cross_entropy_loss", "mse_loss"]

_LOG = get_logger(__name__)


def mse_loss(predictions: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    return F.mse_loss(predictions, targets)


def cross_entropy_loss(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    return F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), targets.reshape(-1))


@dataclass
class StepMetrics:
    step: int
    loss: float
    learning_rate: float
    grad_norm: float | None = None
    seconds: float = 0.0
    forward_seconds: float = 0.0
    backward_seconds: float = 0.0
    samples: int = 0
    skipped: bool = False

    def as_dict(self) -> dict[str, Any]:
        return {"step": self.step, "loss": self.loss, "learning_rate": self.learning_rate, "grad_norm": self.grad_norm,
                "seconds": self.seconds, "forward_seconds": self.forward_seconds, "backward_seconds": self.backward_seconds,
                "samples": self.samples, "skipped": self.skipped}


@dataclass
class TrainingEngine:
    config: ExperimentConfig
    context: DistributedContext
    recorder: CommunicationRecorder | None = None
    model: HybridModel = field(init=False)
    optimizer: ShardedOptimizer = field(init=False)
    scheduler: LearningRateSchedule = field(init=False)
    scaler: GradScaler = field(init=False)
    state: TrainingState = field(init=False)
    history: list[StepMetrics] = field(init=False, default_factory=list)

    def __post_init__(self) -> None:
        cfg, ctx = self.config, self.context
        if self.recorder is None and cfg.training.collect_metrics:
            self.recorder = CommunicationRecorder()
        # Deterministic-algorithm mode is a CPU/Gloo debugging aid; the CUDA path is deterministic by construction
        # except for the atomic-add reductions (embedding and attention dQ), which are order-dependent in the last bits.
        deterministic = cfg.training.deterministic and ctx.device.type == "cpu"
        if ctx.device.type == "cuda":
            from .. import ops

            # Reproducible split-K sums when asked for; otherwise partial tiles are reduce-added in place.
            ops.set_deterministic_reductions(cfg.training.deterministic)
        seed_everything(cfg.training.seed, stream="model-init", deterministic=deterministic)
        ctx.fused_tensor_collectives = bool(cfg.tensor_parallel.fused_collectives and ctx.device.type == "cuda")
        self.model = build_parallel_model(cfg, ctx, recorder=self.recorder)
        seed_everything(cfg.training.seed, stream="runtime", index=ctx.group("dp_shard").local_rank, deterministic=deterministic)
        self.compute_dtype = cfg.mixed_precision.compute_dtype
        self.optimizer = ShardedOptimizer(self.model.optimizer_parameters(), cfg.optimizer, norm_group=self.model.norm_group,
                                          device=ctx.device, recorder=self.recorder,
                                          compute_dtype=self.compute_dtype if cfg.mixed_precision.enabled else None)
        self.scheduler = LearningRateSchedule(cfg.scheduler, base_learning_rate=cfg.optimizer.learning_rate,
                                              total_steps=max(cfg.training.max_steps, 1))
        self.scaler = GradScaler(cfg.mixed_precision.scaler, ctx.group("world"), ctx.device, recorder=self.recorder)
        self._fsdp_fused_update = self._enable_fsdp_fused_update()
        self._overlap = self._enable_overlapped_step()
        self._ddp_flat_base = self._ddp_flat_offset()
        self.state = TrainingState()
        self._transformer = cfg.model.kind == "transformer"
        self._fused_loss = self._transformer and cfg.model.fused_loss
        self._criterion: Callable[[torch.Tensor, torch.Tensor], torch.Tensor] = cross_entropy_loss if self._transformer else mse_loss
        self._build_data()
        self._graph: torch.cuda.CUDAGraph | None = None
        self.graph_enabled = True  # replay the captured step when TrainingConfig.cuda_graph is set
        self._graph_io: dict[str, Any] = {}
        self._eager_steps = 0
        self._graph_done: torch.cuda.Event | None = None
        self.last_loss_tensor: torch.Tensor | None = None
        self.last_grad_norm_tensor: torch.Tensor | None = None
        reset_peak_memory(ctx.device)
        _LOG.info("engine built (%s), %d parameters on this rank", self.model.description.strategy,
                  sum(p.numel() for p in self.model.optimizer_parameters()))

    def _enable_fsdp_fused_update(self) -> bool:
        """Turn on the FSDP reduce-scatter + AdamW kernel when the step does not need the gradients afterwards.

        The fused kernel updates each unit during the backward pass, so it needs: FSDP on CUDA with
        ``fsdp.fused_update``, the fused AdamW optimizer, no clipping, no gradient-norm metric and no
        loss scaling.  Every input is configuration, so every rank decides the same way.
        """
        cfg, ctx = self.config, self.context
        fsdp = self.model.fsdp
        inner = self.optimizer.inner
        if (fsdp is None or ctx.device.type != "cuda" or not cfg.fsdp.fused_update or not isinstance(inner, FusedAdamW)
                or cfg.training.max_grad_norm > 0 or cfg.training.collect_metrics or self.scaler.enabled):
            return False
        workspace = ctx.symmetric_workspace("shard")
        # Hybrid sharding: the replicas' gradients are summed by the same kernel over the
        # data-parallel x shard group.
        reduce_ws = ctx.symmetric_workspace("dp_shard") if ctx.group("data_parallel").size > 1 else None
        return fsdp.enable_fused_update(workspace, inner, accumulate=cfg.training.gradient_accumulation_steps > 1,
                                        reduce_workspace=reduce_ws)

    fsdp_fused_update = property(lambda self: self._fsdp_fused_update)

    def _enable_overlapped_step(self) -> OverlappedAdamW | None:
        """Update each gradient bucket during the backward pass when nothing global is needed first.

        Needs the fused AdamW on CUDA without FSDP (whose reduce-scatter kernel already updates
        during the backward), no clipping, no gradient-norm metric and no loss scaling, and
        ``training.overlap_optimizer_step``.  Every input is configuration, so all ranks agree.
        """
        cfg, ctx = self.config, self.context
        inner = self.optimizer.inner
        if (not cfg.training.overlap_optimizer_step or ctx.device.type != "cuda" or self.model.fsdp is not None
                or not isinstance(inner, FusedAdamW) or not inner.flat_parameters.is_cuda or cfg.training.max_grad_norm > 0
                or cfg.training.collect_metrics or self.scaler.enabled or self.optimizer.offloaded):
            return None
        ddp = self.model.ddp
        if ddp is not None:
            if ddp.flat_gradient_buffer.untyped_storage().data_ptr() != inner.flat_gradients.untyped_storage().data_ptr():
                return None  # the optimizer's flat space does not mirror the buckets
            overlap = OverlappedAdamW(inner, track_parameters=False)
            ddp.post_reduction_hook = overlap.bucket_reduced
            return overlap
        return OverlappedAdamW(inner, group_bytes=int(cfg.ddp.bucket_cap_mb * (1 << 20)))

    overlapped_step = property(lambda self: self._overlap)

    def _ddp_flat_offset(self) -> int | None:
        """Index in the fused optimizer's flat buffers of DDP's flat gradient buffer start, or ``None``
        when the two do not share storage (then no bucket's update can be deferred)."""
        ddp = self.model.ddp
        inner = self.optimizer.inner
        if (ddp is None or self.context.device.type != "cuda" or not isinstance(inner, FusedAdamW)
                or not inner.flat_parameters.is_cuda or self.optimizer.offloaded):
            return None
        buf, flat = ddp.flat_gradient_buffer, inner.flat_gradients
        if buf.untyped_storage().data_ptr() != flat.untyped_storage().data_ptr():
            return None
        return int(buf.storage_offset() - flat.storage_offset())

    # -- data ----------------------------------------------------------------------------------------------
    def _build_data(self) -> None:
        cfg = self.config
        group = self.model.data_group
        train = build_dataset(cfg.model, cfg.data, split="train")
        self.train_sampler = DistributedBatchSampler(len(train), cfg.data.micro_batch_size, group, shuffle=cfg.data.shuffle,
                                                     seed=cfg.data.seed)
        self.train_loader = SyntheticDataLoader(train, self.train_sampler, self.context.device)
        self.eval_loader: SyntheticDataLoader | None = None
        if cfg.data.num_eval_samples > 0:
            ev = build_dataset(cfg.model, cfg.data, split="eval")
            self.eval_loader = SyntheticDataLoader(ev, DistributedBatchSampler(len(ev), cfg.data.micro_batch_size, group,
                                                                               shuffle=False, seed=cfg.data.seed), self.context.device)
        need = cfg.training.gradient_accumulation_steps
        if len(self.train_loader) < need:
            raise ConfigurationError(format_error(
                "engine.build_data", "the training set yields fewer micro-batches in one epoch than one step consumes",
                rank=self.context.rank, world_size=self.context.world_size, expected=f">= {need} micro-batches in one epoch",
                observed=len(self.train_loader), resolution="raise data.num_train_samples or lower gradient_accumulation_steps"))

    def batch_stream(self, *, host: bool = False) -> Any:
        """Endless stream of this rank's micro-batches (on the device, or pinned host memory with ``host``)."""
        while True:
            epoch = self.state.epoch
            source = self.train_loader.iter_host(epoch) if host else self.train_loader.iter_epoch(epoch)
            for i, batch in enumerate(source):
                if i < self.state.batches_in_epoch:
                    continue
                self.state.batches_in_epoch = i + 1
                yield batch
            self.state.epoch += 1
            self.state.batches_in_epoch = 0

    # -- the loop ---------------------------------------------------------------------------------------------
    def train(self, max_steps: int | None = None) -> TrainingState:
        target = self.config.training.max_steps if max_steps is None else max_steps
        batches = self.batch_stream(host=self._use_graph())
        while self.state.step < target:
            m = self.train_step(batches)
            self.history.append(m)
            t = self.config.training
            if t.log_every_steps > 0 and self.state.step % t.log_every_steps == 0:
                _LOG.info("[%d/%d] loss %.6f | lr %.3e | grad-norm %s | %.3f s", self.state.step, target, m.loss, m.learning_rate,
                          "n/a" if m.grad_norm is None else f"{m.grad_norm:.4f}", m.seconds, extra={"primary_only": True})
            if t.eval_every_steps > 0 and self.state.step % t.eval_every_steps == 0:
                self.state.best_eval_loss = min(self.state.best_eval_loss, self.evaluate())
            if self.config.checkpoint.save_every_steps > 0 and self.state.step % self.config.checkpoint.save_every_steps == 0:
                self.save_checkpoint()
        return self.state

    def _use_graph(self) -> bool:
        return bool(self.config.training.cuda_graph and self.graph_enabled and self.context.device.type == "cuda")

    def _loss(self, inputs: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        if self._fused_loss:
            return self.model(inputs, targets=targets)
        return self._criterion(self.model(inputs), targets)

    def _device_step(self, micro_batches: list[tuple[torch.Tensor, torch.Tensor]]) -> tuple[torch.Tensor, torch.Tensor | None]:
        """Forward/backward/reduce/clip/update with no host synchronisation; returns device (loss, grad norm)."""
        n = len(micro_batches)
        total = None
        inner = self.optimizer.inner
        if self._fsdp_fused_update:
            # The update runs inside the backward pass's reduce-scatter kernels: stage [lr, step, ...] first.
            inner.stage_hyper_parameters()
        if self._overlap is not None:
            self._overlap.begin()
        for i, (x, y) in enumerate(micro_batches):
            ctx = self.model.no_sync() if i < n - 1 else _null()
            armed = self._overlap.armed() if (self._overlap is not None and i == n - 1) else _null()
            with ctx:
                with trace_range(f"step/forward {i}"):
                    loss = self._loss(x, y) / n
                with trace_range(f"step/backward {i}"), armed:
                    self.scaler.scale(loss).backward()
            total = loss.detach() if total is None else total + loss.detach()
        t = self.config.training
        # Plain fused AdamW after DDP's in-kernel all-reduce: update every other bucket while the
        # last one (reduced only after the backward pass) is still on the wire.
        split = (self._overlap is None and not self._fsdp_fused_update and self._ddp_flat_base is not None
                 and not self.scaler.enabled and not (t.max_grad_norm > 0 or t.collect_metrics))
        with trace_range("step/finish_backward"):
            deferred = self.model.finish_backward(defer_last=split)
        if deferred is not None:
            deferred = (deferred[0] + self._ddp_flat_base, deferred[1], deferred[2])
        params = self.model.optimizer_parameters()
        if self.scaler.enabled:
            self.scaler.unscale_(params)
        norm = None
        if t.max_grad_norm > 0 or t.collect_metrics:
            norm = self.optimizer.clip_grad_norm(t.max_grad_norm)
        if self._fsdp_fused_update:
            pass  # every flat shard was updated by its unit's reduce-scatter kernel
        elif self._overlap is not None:
            ddp = self.model.ddp
            self._overlap.finish(ddp.communication_stream if ddp is not None else None)
        elif isinstance(inner, FusedAdamW) and inner.flat_parameters.is_cuda and not self.scaler.enabled:
            with trace_range("step/adamw"):
                inner.launch_step(deferred)
        elif self.scaler.enabled:
            self.scaler.step(self.optimizer, params, already_unscaled=True)
        else:
            self.optimizer.step()
        self.optimizer.zero_grad(set_to_none=True)
        group = self.model.metric_group
        reduced = total.reshape(1).float().clone()
        all_reduce(reduced, group, op=ReduceOp.AVG, recorder=self.recorder).wait()
        return reduced, norm

    def train_step(self, batches: Any, *, read_metrics: bool = True) -> StepMetrics:
        """One optimizer step; ``batches`` yields :class:`Batch` objects (on the device, or pinned host for graphs)."""
        start = time.perf_counter()
        n = self.config.training.gradient_accumulation_steps
        lr = self.scheduler.value_at(self.state.step)
        self.optimizer.set_learning_rate(lr)
        micro = [next(batches) for _ in range(n)]
        samples = sum(b.size for b in micro)
        inner = self.optimizer.inner
        if self._graph_done is not None:
            # The captured step reads the optimizer's pinned hyper-parameter buffer; do not
            # overwrite it before the previous replay has consumed it.
            self._graph_done.synchronize()
        if isinstance(inner, FusedAdamW) and inner.flat_parameters.is_cuda and not self.scaler.enabled:
            inner.prepare_step()
        if self._use_graph():
            loss_t, norm_t = self._graph_step(micro)
        else:
            dev = self.context.device
            pairs = [(b.inputs.to(dev, non_blocking=True), b.targets.to(dev, non_blocking=True)) for b in micro]
            loss_t, norm_t = self._device_step(pairs)
        self.last_loss_tensor, self.last_grad_norm_tensor = loss_t, norm_t
        skipped = self.scaler.enabled and self.scaler.last_step_skipped
        if self.scaler.enabled:
            self.scaler.update()
        global_samples = samples * self.model.data_group.size
        if skipped:
            self.state.step += 1
            self.state.skipped_steps += 1
            self.state.samples_seen += global_samples
        else:
            self.state.advance_step(samples=global_samples)
        loss, norm = float("nan"), None
        if read_metrics:
            loss, norm = self.read_step_results(loss_t, norm_t)
        self.state.last_loss = loss
        return StepMetrics(self.state.step, loss, lr, norm, time.perf_counter() - start, samples=global_samples, skipped=skipped)

    def read_step_results(self, loss_t: torch.Tensor, norm_t: torch.Tensor | None) -> tuple[float, float | None]:
        """Loss, gradient norm and the status words of every in-kernel collective, in one device-to-host read.

        The status words are written by bounded waits inside the NVLink kernels (DDP bucket
        all-reduce, FSDP reduce-scatter + AdamW, tensor-parallel GEMM collectives), also when the step
        was replayed from a CUDA graph; a non-zero word raises :class:`KernelError` here, so a step
        whose reduction gave up on a peer never passes as a normal one.
        """
        parts = [loss_t.detach().reshape(1).float()]
        if norm_t is not None:
            parts.append(norm_t.detach().reshape(1).float())
        workspaces = self.context.symmetric_workspaces() if self.context.device.type == "cuda" else []
        parts += [ws.status[:1].float() for ws in workspaces]
        host = torch.cat(parts).cpu() if len(parts) > 1 else parts[0].cpu()
        codes = host[len(parts) - len(workspaces):].tolist()
        for ws, code in zip(workspaces, codes):
            if code != 0:
                ws.check_status()  # raises KernelError with the stage that gave up
        loss = float(host[0])
        norm = float(host[1]) if norm_t is not None else None
        return loss, norm

    # -- CUDA graph -------------------------------------------------------------------------------------------------
    def _graph_step(self, micro: list[Batch]) -> tuple[torch.Tensor, torch.Tensor | None]:
        io = self._graph_io
        if not io:
            io["inputs"] = [torch.empty_like(b.inputs, device=self.context.device) for b in micro]
            io["targets"] = [torch.empty_like(b.targets, device=self.context.device) for b in micro]
        for dst, b in zip(io["inputs"], micro):
            dst.copy_(b.inputs, non_blocking=True)
        for dst, b in zip(io["targets"], micro):
            dst.copy_(b.targets, non_blocking=True)
        pairs = list(zip(io["inputs"], io["targets"]))
        if self._graph is None:
            # Warm up eagerly on a side stream (allocator pools, lazy inits, NCCL communicators), then capture.
            if self._eager_steps < 2:
                self._eager_steps += 1
                return self._device_step(pairs)
            stream = torch.cuda.Stream()
            stream.wait_stream(torch.cuda.current_stream())
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(graph, stream=stream):
                    loss, norm = self._device_step(pairs)
            torch.cuda.current_stream().wait_stream(stream)
            io["loss"], io["norm"] = loss, norm
            self._graph = graph
        self._graph.replay()
        if self._graph_done is None:
            self._graph_done = torch.cuda.Event()
        self._graph_done.record()
        return self._graph_io["loss"], self._graph_io["norm"]

    def release_graph(self) -> None:
        """Drop the captured graph (required before destroying process groups it uses)."""
        self._graph = None
        self._graph_io.clear()
        self._graph_done = None

    # -- evaluation / checkpoints --------------------------------------------------------------------------------------------
    @torch.no_grad()
    def evaluate(self) -> float:
        if self.eval_loader is None:
            return float("nan")
        was_training = self.model.training
        self.model.eval()
        total, count = 0.0, 0
        for batch in self.eval_loader.iter_epoch(0):
            total += float(self._loss(batch.inputs, batch.targets).item())
            count += 1
        if was_training:
            self.model.train()
        loss = self.model.reduce_metric(total / max(count, 1))
        _LOG.info("evaluation at step %d: loss %.6f", loss, self.state.step, extra={"primary_only": True})
        return loss

    def save_checkpoint(self, directory: str | Path | None = None) -> Path:
        from ..checkpoint.writer import save_checkpoint

        root = Path(directory) if directory is not None else Path(self.config.checkpoint.directory)
        result = save_checkpoint(root, model=self.model, context=self.context, state=self.state, optimizer=self.optimizer,
                                 config=self.config, scheduler_state=self.scheduler.state_dict(),
                                 scaler_state=self.scaler.state_dict(),
                                 extra_metadata={"batches_in_epoch": self.state.batches_in_epoch,
                                                 "dataset_size": len(self.train_loader.dataset),
                                                 "micro_batch_size": self.config.data.micro_batch_size},
                                 save_optimizer=self.config.checkpoint.save_optimizer_state,
                                 save_rng=self.config.checkpoint.save_rng_state, keep_last=self.config.checkpoint.keep_last)
        return result.path

    def load_checkpoint(self, directory: str | Path | None = None) -> LoadedCheckpoint:
        from ..checkpoint.reader import load_checkpoint
        from ..checkpoint.writer import find_latest_checkpoint

        if directory is not None:
            target: Path | None = Path(directory)
        elif self.config.checkpoint.resume_from:
            target = Path(self.config.checkpoint.resume_from)
        else:
            target = find_latest_checkpoint(self.config.checkpoint.directory)
        if target is None:
            raise ConfigurationError(format_error("engine.load_checkpoint", "there is no checkpoint to resume", rank=self.context.rank,
                                                  world_size=self.context.world_size, expected="a directory holding a published checkpoint",
                                                  observed=self.config.checkpoint.directory,
                                                  resolution="name the checkpoint directory, or set checkpoint.resume_from"))
        result = load_checkpoint(target, model=self.model, context=self.context, optimizer=self.optimizer, config=self.config,
                                 verify_checksums=self.config.checkpoint.verify_checksums_on_load,
                                 load_optimizer=self.config.checkpoint.save_optimizer_state,
                                 load_rng=self.config.checkpoint.save_rng_state)
        self.optimizer.refresh_compute_copies()
        self.state = replace(result.state)
        if result.scheduler_state:
            self.scheduler = LearningRateSchedule.from_state_dict(result.scheduler_state)
        if result.scaler_state:
            self.scaler.load_state_dict(result.scaler_state)
        extra = result.metadata.get("extra", {})
        if "batches_in_epoch" in extra:
            self.state.batches_in_epoch = int(extra["batches_in_epoch"])
        return result

    def memory_snapshot(self) -> MemorySnapshot:
        return capture_memory(self.context.device, include_gc_scan=True)

    def communication_summary(self) -> str:
        if self.recorder is None:
            return "collectives are not being counted; set training.collect_metrics to record them"
        return self.recorder.summary()

    def parameter_count(self) -> dict[str, int]:
        local = sum(p.numel() for p in self.model.optimizer_parameters())
        return {"local": local, "global": int(sum_scalar(float(local), self.context.group("world"), device=self.context.device))}

    def close(self) -> None:
        self.release_graph()
        if self._overlap is not None:
            self._overlap.close()
        if self.model.ddp is not None:
            self.model.ddp.teardown()


class _null:
    def __enter__(self) -> None:
        return None

    def __exit__(self, *exc: object) -> None:
        return None
