"""Composition of all strategies over the 4-D grid, and the rendered parallel plan.

Same rules as ``src/hybrid_training/parallel/hybrid.py:120-848``:

* ``shard > 1`` wraps the model in FSDP over the shard group, with the data
  group as the replica group (HSDP) when ``data_parallel > 1``;
* otherwise ``data_parallel > 1`` wraps it in DDP;
* tensor / sequence parallelism live inside the model's layers;
* metrics are averaged over ``dp_shard``; the gradient norm is reduced over
  ``world`` with per-parameter multiplicity weights;
* tensor-parallel slices are stored under ``name#tp{K}of{N}``.

One ordering differs: the sequence-parallel partial gradients are summed
*after* DDP's bucket all-reduce, on the synchronised bucket views (both are
linear, so the order does not change the result; doing it afterwards means the
SP sum acts on the buffer that the optimizer will read).  Under FSDP the SP sum
happens inside each unit before its reduce-scatter.
"""

from __future__ import annotations

from collections.abc import Iterator
from contextlib import AbstractContextManager, contextmanager, nullcontext
from dataclasses import dataclass, field
from typing import Any

import torch
import torch.nn as nn

from ..config import ExperimentConfig
from ..distributed.collectives import CommunicationRecorder, ReduceOp, assert_tensor_consistent, sum_scalar
from ..distributed.context import DistributedContext
from ..distributed.groups import GroupHandle
from ..errors import ConfigurationError, ShardingError, format_error
from ..logging import get_logger
from .ddp import DistributedDataParallel
from .fsdp import FullyShardedDataParallel, PieceLayout, ShardedTensorPiece
from .tensor_parallel import all_reduce_sequence_parallel_gradients

__all__ = ["HybridModel", "ParallelismDescription", "PlanStep", "ParameterParallelInfo", "build_model", "build_parallel_model",
           "describe_parallel_plan"]

_LOG = get_logger(__name__)


@dataclass(frozen=True)
class ParameterParallelInfo:
    name: str
    shape: tuple[int, ...]
    partition_dim: int | None
    tensor_parallel_size: int
    tensor_parallel_rank: int

    @property
    def storage_key(self) -> str:
        """Checkpoint key: the name, plus ``#tp{rank}of{size}`` for tensor-parallel slices."""
        if self.tensor_parallel_size <= 1:
            return self.name
        return f"{self.name}#tp{self.tensor_parallel_rank}of{self.tensor_parallel_size}"

    def as_dict(self) -> dict[str, Any]:
        return {"name": self.name, "shape": list(self.shape), "partition_dim": self.partition_dim,
                "tensor_parallel_size": self.tensor_parallel_size, "tensor_parallel_rank": self.tensor_parallel_rank}


@dataclass(frozen=True)
class PlanStep:
    """One collective of the training step: when it runs, what it moves, over which group, and by which code."""

    phase: str           # "forward", "backward", "optimizer" or "metrics"
    operation: str       # what is communicated
    group: str           # process-group name of the 4-D grid
    implementation: str  # the kernel or library call that performs it on this configuration


@dataclass
class ParallelismDescription:
    """The parallel plan of one rank: placement of parameters / activations and every collective of a step.

    ``steps`` lists the collectives in the order a step issues them, each with the implementation
    this configuration selects (in-kernel NVLink collective, NCCL, or Gloo).  The list fields
    summarise the same plan by group for programmatic checks.
    """

    strategy: str
    replicated_parameters: list[str] = field(default_factory=list)
    sharded_parameters: list[str] = field(default_factory=list)
    sharded_activations: list[str] = field(default_factory=list)
    gradient_reductions: list[tuple[str, str]] = field(default_factory=list)
    metric_group: str = "dp_shard"
    notes: list[str] = field(default_factory=list)
    steps: list[PlanStep] = field(default_factory=list)

    def render(self) -> str:
        width = max([len(s.operation) for s in self.steps] + [9])
        out = [f"plan: {self.strategy}",
               f"  weights   replicated over {', '.join(self.replicated_parameters) or 'nothing'}; "
               f"split over {', '.join(self.sharded_parameters) or 'nothing'}",
               f"  activations split over {', '.join(self.sharded_activations) or 'nothing'}",
               f"  loss / metrics averaged over {self.metric_group}"]
        for phase in ("forward", "backward", "optimizer", "metrics"):
            rows = [s for s in self.steps if s.phase == phase]
            if rows:
                out.append(f"  {phase}:")
                out += [f"    {s.operation:<{width}}  [{s.group}]  {s.implementation}" for s in rows]
        out += [f"  * {n}" for n in self.notes]
        return "\n".join(out)


def build_model(config: ExperimentConfig, context: DistributedContext, *, device: torch.device | None = None) -> nn.Module:
    """Instantiate the configured model with this rank's tensor/sequence-parallel plan."""
    from ..models.mlp import MLP
    from ..models.transformer import ParallelPlan, TinyTransformer

    device = device if device is not None else context.device
    tensor = context.group("tensor")
    sequence = context.group("sequence_effective")
    sp = config.topology.sequence_parallel_enabled
    if config.model.kind == "transformer":
        if device.type == "cuda" and config.mixed_precision.compute_dtype != torch.bfloat16:
            raise ConfigurationError(format_error(
                "hybrid.build_model", "the transformer's CUDA kernels (tcgen05 GEMMs, attention, fused norms) compute in "
                "bf16 with fp32 master weights", rank=context.rank, world_size=context.world_size,
                expected="mixed_precision.enabled=True with param_dtype='bfloat16' on CUDA",
                observed=str(config.mixed_precision.compute_dtype),
                resolution="enable bf16 mixed precision (fp32 compute is available on the CPU path)"))
        plan = ParallelPlan(tensor_group=tensor, sequence_group=sequence, sequence_parallel=sp, vocab_parallel=tensor.size > 1,
                            ring_attention=config.tensor_parallel.context_parallel_algorithm == "ring",
                            ulysses_attention=config.tensor_parallel.context_parallel_algorithm == "ulysses")
        return TinyTransformer(config.model, plan, seed=config.training.seed, device=device,
                               compute_dtype=config.mixed_precision.compute_dtype)
    if sp:
        raise ConfigurationError(format_error("hybrid.build_model", "the MLP has no sequence dimension to split",
                                              rank=context.rank, world_size=context.world_size,
                                              expected="a transformer model (sequence parallelism splits its tokens)",
                                              observed=config.model.kind, resolution="use the transformer or disable SP"))
    return MLP(config.model, seed=config.training.seed, tensor_parallel_group=tensor if tensor.size > 1 else None, device=device)


def describe_parallel_plan(config: ExperimentConfig, context: DistributedContext) -> ParallelismDescription:
    """Which rank holds what, and which collective (and which implementation of it) each step runs.

    The implementations named are the ones this framework selects for ``config`` on this
    context's device: in-kernel NVLink collectives (``ops/csrc/comm.cu``, the collective mode of
    ``ops/csrc/gemm_tcgen05.cu``) on CUDA when their switches are on and the group has a
    peer-mapped workspace, otherwise the process group's backend (NCCL on CUDA, Gloo on CPU).
    """
    topo = context.topology
    dp, shard, tp = topo.size("data_parallel"), topo.size("shard"), topo.size("tensor")
    sp = topo.sequence_parallel_enabled
    independent = sp and config.topology.sequence_parallel_mode == "independent"
    cuda = context.device.type == "cuda"
    library = "NCCL" if cuda else "Gloo"
    parts = [name for name, on in (("fsdp", shard > 1), ("hsdp-replicas" if shard > 1 else "ddp", dp > 1),
                                   ("tp", tp > 1), ("context-parallel" if independent else "sp", sp)) if on]
    plan = ParallelismDescription(strategy=" x ".join(parts) if parts else "single-process")
    if tp > 1:
        plan.sharded_parameters.append("tensor")
    if shard > 1:
        plan.sharded_parameters.append("shard")
    if dp > 1:
        plan.replicated_parameters.append("data_parallel")
    if sp:
        plan.sharded_activations.append(topo.sequence_group_name)
    add = plan.steps.append

    fused_tp = cuda and config.tensor_parallel.fused_collectives
    if tp > 1:
        add(PlanStep("forward", "vocab-parallel embedding partial rows", "tensor",
                     f"{library} {'reduce-scatter' if sp else 'all-reduce'} after the masked gather kernel"))
        if sp:
            add(PlanStep("forward", "sequence all-gather into column-parallel GEMMs (fused QKV, gate/up)", "tensor",
                         "all-gather inside the tcgen05 GEMM's operand loads" if fused_tp else f"{library} all-gather"))
            add(PlanStep("forward", "row-parallel GEMM output to sequence shards", "tensor",
                         "reduce-scatter in the tcgen05 GEMM epilogue" if fused_tp else f"{library} reduce-scatter"))
        else:
            add(PlanStep("forward", "row-parallel GEMM partial sums", "tensor",
                         "fp32 partials written by the GEMM into peer memory, summed by the in-kernel NVLink all-reduce"
                         if fused_tp else f"{library} all-reduce"))
        add(PlanStep("forward", "vocab-parallel cross-entropy statistics (max, sum-exp, target logit)", "tensor",
                     f"{library} all-reduce of 3 floats per token; no logits are gathered"))
        add(PlanStep("backward", "column-parallel input gradients", "tensor",
                     ("reduce-scatter in the data-gradient GEMM epilogue" if fused_tp else f"{library} reduce-scatter")
                     if sp else ("fp32 partials written by the data-gradient GEMM into peer memory, summed by the in-kernel "
                                 "NVLink all-reduce" if fused_tp else f"{library} all-reduce")))
    if independent:
        algorithm = config.tensor_parallel.context_parallel_algorithm
        add(PlanStep("forward", "attention keys / values" if algorithm != "ulysses" else "attention sequence <-> head re-shard",
                     topo.sequence_group_name,
                     {"ring": f"{library} send/recv ring with online-softmax merge",
                      "ulysses": f"{library} all-to-all to head groups, flash attention over the whole sequence, all-to-all back"}
                     .get(algorithm, f"{library} all-gather")))
    if shard > 1:
        fused_fsdp = cuda and config.fsdp.fused_update
        add(PlanStep("forward", "flat-parameter all-gather per unit", "shard",
                     "peer copies of bf16 shards (copy engines, prefetching the next unit)" if fused_fsdp
                     else f"{library} all-gather"))
        if config.fsdp.reshard_after_forward:
            add(PlanStep("backward", "flat-parameter re-gather per unit", "shard",
                         "peer copies of bf16 shards" if fused_fsdp else f"{library} all-gather"))
        if dp > 1 and fused_fsdp and shard * dp <= 8:
            add(PlanStep("backward", "flat-gradient reduce-scatter per unit, summed across replicas", "dp_shard",
                         "one kernel over the replicas x shards: every replica's slice summed over peer memory + 1/(G R) + "
                         "AdamW on the shard, when the step needs no global gradient norm or loss scaling; otherwise "
                         f"{library} reduce-scatter, then {library} all-reduce across replicas"))
        else:
            add(PlanStep("backward", "flat-gradient reduce-scatter per unit", "shard",
                         "one kernel: reduce-scatter over peer memory + 1/G + AdamW on the shard, when the step needs no "
                         "global gradient norm or loss scaling; otherwise " + library if fused_fsdp else f"{library} reduce-scatter"))
            if dp > 1:
                add(PlanStep("backward", "sharded-gradient all-reduce across replicas", "data_parallel", f"{library} all-reduce"))
    elif dp > 1:
        add(PlanStep("backward", f"gradient buckets of {config.ddp.bucket_cap_mb:g} MiB, launched in bucket order",
                     "data_parallel",
                     "in-kernel NVLink all-reduce with 1/G folded in, on a high-priority stream overlapping the backward"
                     if cuda and config.ddp.fused_allreduce else f"{library} all-reduce of pre-scaled buckets"))
    if sp and not independent and shard == 1:
        add(PlanStep("backward", "sequence-parallel partial gradients (norm weights, row biases)", "tensor",
                     f"{library} all-reduce after the data-parallel buckets"))
    if config.training.max_grad_norm > 0 or config.training.collect_metrics:
        add(PlanStep("optimizer", "weighted squared gradient norm", "world",
                     f"device-side sum of squares, {library} all-reduce of one scalar, no host read"))
    add(PlanStep("metrics", "step loss", "dp_shard", f"{library} all-reduce of one scalar"))

    for s in plan.steps:
        if s.phase == "backward" and ("gradient" in s.operation) and s.group != "tensor":
            plan.gradient_reductions.append((s.operation, s.group))
    if tp > 1 or sp:
        plan.notes.append("every rank of a tensor group must see the same token batch (the sampler slices by dp_shard only)")
    if shard > 1 and dp > 1:
        plan.notes.append(f"parameters and optimizer state are divided by shard={shard} only; the {dp} replicas each hold "
                          "a full set of shards")
    if shard > 1 and config.fsdp.auto_wrap_min_num_params == 0:
        plan.notes.append("no auto-wrap threshold: the model is a single FSDP unit and its gathered copy is full size")
    if config.training.gradient_accumulation_steps > 1:
        plan.notes.append(f"{config.training.gradient_accumulation_steps} micro-batches per step: gradient collectives run "
                          "after the last one only")
    if config.training.cuda_graph and cuda:
        plan.notes.append("the step (forward, backward, reductions, update) is replayed as one captured CUDA graph")
    return plan


def _unique_named_parameters(model: nn.Module) -> dict[str, nn.Parameter]:
    seen: set[int] = set()
    out: dict[str, nn.Parameter] = {}
    for name, p in model.named_parameters():
        if id(p) not in seen:
            seen.add(id(p))
            out[name] = p
    return out


class HybridModel(nn.Module):
    """The model wrapped for the grid: FSDP / DDP / plain, plus SP gradient handling and state views."""

    def __init__(self, model: nn.Module, config: ExperimentConfig, context: DistributedContext, *,
                 recorder: CommunicationRecorder | None = None) -> None:
        super().__init__()
        self._config, self._context, self._recorder = config, context, recorder
        self._description = describe_parallel_plan(config, context)
        shard, replica = context.group("shard"), context.group("data_parallel")
        sp = config.topology.sequence_parallel_enabled
        self._sp_group: GroupHandle | None = context.group("sequence_effective") if sp else None
        self._fsdp: FullyShardedDataParallel | None = None
        self._ddp: DistributedDataParallel | None = None
        if shard.size > 1:
            self._fsdp = FullyShardedDataParallel(model, shard, config.fsdp, replica_group=replica if replica.size > 1 else None,
                                                  mixed_precision=config.mixed_precision, device=context.device,
                                                  recorder=recorder, sequence_group=self._sp_group)
            self.wrapped: nn.Module = self._fsdp
        elif replica.size > 1:
            workspace = None
            if config.ddp.fused_allreduce and context.device.type == "cuda":
                workspace = context.symmetric_workspace("data_parallel")
            self._ddp = DistributedDataParallel(model, replica, config.ddp, recorder=recorder, workspace=workspace)
            self.wrapped = self._ddp
        else:
            self.wrapped = model
        self._inner_model = model
        _LOG.info("hybrid model ready\n%s", self._description.render())

    def forward(self, *args: Any, **kwargs: Any) -> Any:
        return self.wrapped(*args, **kwargs)

    def no_sync(self) -> AbstractContextManager[None]:
        if self._ddp is not None:
            return self._ddp.no_sync()
        if self._fsdp is not None:
            return self._fsdp.no_sync()
        return nullcontext()

    def finish_backward(self, *, defer_last: bool = False) -> tuple[int, int, Any] | None:
        """Complete every gradient reduction for the step (DDP wait, SP partial sums, FSDP free).

        ``defer_last``: with DDP's in-kernel all-reduce and no sequence-parallel partial sums, leave
        the last bucket's reduction running and return ``(start, numel, wait)`` for it (see
        :meth:`DistributedDataParallel.finish_gradient_synchronization`).
        """
        if self._ddp is not None:
            deferred = self._ddp.finish_gradient_synchronization(defer_last=defer_last and self._sp_group is None)
            if deferred is not None:
                return deferred
        if self._sp_group is not None and self._fsdp is None:
            all_reduce_sequence_parallel_gradients(self._inner_model, self._sp_group, recorder=self._recorder)
        if self._fsdp is not None:
            self._fsdp.finish_backward()
        return None

    def optimizer_parameters(self) -> list[nn.Parameter]:
        return [p for p in self.wrapped.parameters() if p.requires_grad]

    metric_group = property(lambda self: self._context.group("dp_shard"))
    norm_group = property(lambda self: self._context.group("world"))
    data_group = property(lambda self: self._context.group("dp_shard"))
    description = property(lambda self: self._description)
    fsdp = property(lambda self: self._fsdp)
    ddp = property(lambda self: self._ddp)
    inner_model = property(lambda self: self._inner_model)

    def reduce_metric(self, value: float | torch.Tensor, *, average: bool = True) -> float:
        return sum_scalar(value, self.metric_group, device=self._context.device,
                          op=ReduceOp.AVG if average else ReduceOp.SUM, recorder=self._recorder)

    def validate_input_replication(self, batch: torch.Tensor) -> None:
        group = self._context.group("tensor_sequence")
        if group.size > 1:
            data = batch.detach().double() if batch.is_floating_point() else batch.detach()
            assert_tensor_consistent(data, group, name="the input batch", operation="hybrid.validate_input_replication")

    def parameter_parallel_info(self) -> dict[str, ParameterParallelInfo]:
        tensor = self._context.group("tensor")
        if self._fsdp is not None:
            described = self._fsdp.original_named_parameters()
        else:
            described = {n: (tuple(p.shape), p) for n, p in _unique_named_parameters(self._inner_model).items()}
        out = {}
        for name, (shape, p) in described.items():
            replicated = bool(getattr(p, "is_tensor_parallel_replicated", True))
            dim = None if replicated else int(getattr(p, "tensor_parallel_partition_dim", 0))
            out[name] = ParameterParallelInfo(name, shape, dim, tensor.size, tensor.local_rank)
        return out

    def optimizer_parameter_layout(self) -> list[list[PieceLayout]]:
        params = self.optimizer_parameters()
        if self._fsdp is not None:
            pairs = self._fsdp.optimizer_parameter_layout()
            if [id(p) for p, _ in pairs] != [id(p) for p in params]:
                raise ShardingError(format_error("hybrid.optimizer_parameter_layout",
                                                 "the FSDP flat-parameter order does not match the optimizer's parameters",
                                                 rank=self._context.rank, expected=len(params), observed=len(pairs),
                                                 resolution="create the optimizer over model.optimizer_parameters()"))
            return [layout for _, layout in pairs]
        by_id = {id(p): (n, tuple(p.shape)) for n, p in _unique_named_parameters(self._inner_model).items()}
        out = []
        for p in params:
            entry = by_id.get(id(p))
            if entry is None:
                raise ShardingError(format_error("hybrid.optimizer_parameter_layout",
                                                 "the optimizer holds a tensor that is not a parameter of this model", rank=self._context.rank,
                                                 expected="one of the model's own parameters", observed=f"tensor {tuple(p.shape)}",
                                                 resolution="create the optimizer over model.optimizer_parameters()"))
            out.append([PieceLayout(entry[0], entry[1], 0, p.numel(), 0)])
        return out

    def sharded_state_dict(self) -> dict[str, ShardedTensorPiece]:
        if self._fsdp is not None:
            return self._fsdp.sharded_state_dict()
        return {n: ShardedTensorPiece(n, tuple(p.shape), 0, p.detach().reshape(-1).clone())
                for n, p in _unique_named_parameters(self._inner_model).items()}

    def buffers_state_dict(self) -> dict[str, torch.Tensor]:
        if self._fsdp is not None:
            return {n: b.detach().clone() for n, b in self._fsdp.original_named_buffers()}
        return {n: b.detach().clone() for n, b in self._inner_model.named_buffers()}

    def full_state_dict(self) -> dict[str, torch.Tensor]:
        if self._fsdp is not None:
            return self._fsdp.full_state_dict()
        out = {n: p.detach().clone() for n, p in _unique_named_parameters(self._inner_model).items()}
        out.update(self.buffers_state_dict())
        return out

    def load_full_state_dict(self, state_dict: dict[str, torch.Tensor]) -> None:
        if self._fsdp is not None:
            self._fsdp.load_full_state_dict(state_dict)
            return
        with torch.no_grad():
            for n, p in _unique_named_parameters(self._inner_model).items():
                if n in state_dict:
                    p.data.copy_(state_dict[n].to(device=p.device, dtype=p.dtype))
            for n, b in self._inner_model.named_buffers():
                if n in state_dict:
                    b.data.copy_(state_dict[n].to(b.dtype))

    @contextmanager
    def summon_full_params(self) -> Iterator[None]:
        if self._fsdp is None:
            yield
            return
        with self._fsdp.summon_full_params():
            yield

    def memory_summary(self) -> dict[str, int]:
        if self._fsdp is not None:
            return self._fsdp.memory_summary()
        params = list(self._inner_model.parameters())
        pb = sum(p.numel() * p.element_size() for p in params)
        gb = sum(p.grad.numel() * p.grad.element_size() for p in params if p.grad is not None)
        return {"shard_bytes": pb, "full_bytes": pb, "grad_shard_bytes": gb, "padding_bytes": 0, "units": 0}

    def __repr__(self) -> str:
        return f"HybridModel({self._description.strategy}, wrapped={type(self.wrapped).__name__})"


def build_parallel_model(config: ExperimentConfig, context: DistributedContext, *, recorder: CommunicationRecorder | None = None,
                         device: torch.device | None = None) -> HybridModel:
    return HybridModel(build_model(config, context, device=device), config, context, recorder=recorder)
