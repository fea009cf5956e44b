"""Structured configuration: frozen dataclasses validated at construction time.

The schema is a strict superset of the reference's
(``src/hybrid_training/config.py:127-1287``): every YAML file written for the
reference loads unchanged, and unknown keys are rejected with their dotted path.
Fields added by this framework (all with defaults that keep the reference
behaviour unless noted):

* ``ModelConfig.norm`` (``layernorm`` | ``rmsnorm``), ``position_embedding``
  (``learned`` | ``rope``), ``rope_theta``, ``num_kv_heads`` (GQA), ``bias``,
  ``activation='swiglu'``, ``fused_loss`` (the head computes a vocab-parallel
  cross-entropy instead of returning gathered logits), ``init_std``.
* ``DataConfig.token_distribution`` (``recurrence`` | ``uniform``).
* ``DDPConfig.fused_allreduce`` / ``TensorParallelConfig.fused_collectives``:
  choose the in-kernel NVLink collective over the NCCL call where the job runs on
  CUDA with symmetric memory available.
* ``TrainingConfig.cuda_graph``: capture the steady-state step in a CUDA graph.
"""

from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass, field, fields, is_dataclass
from pathlib import Path
from typing import Any, TypeVar, Union, get_args, get_origin

import torch
import yaml

from .errors import ConfigurationError, TopologyError, format_error

__all__ = [
    "CheckpointConfig",
    "DDPConfig",
    "DataConfig",
    "ExperimentConfig",
    "FSDPConfig",
    "GradScalerConfig",
    "MixedPrecisionConfig",
    "ModelConfig",
    "OptimizerConfig",
    "SchedulerConfig",
    "SequenceParallelMode",
    "TensorParallelConfig",
    "TopologyConfig",
    "TrainingConfig",
    "load_experiment_config",
    "resolve_dtype",
]

_DTYPE_NAMES: dict[str, torch.dtype] = {
    "float32": torch.float32,
    "fp32": torch.float32,
    "float64": torch.float64,
    "fp64": torch.float64,
    "float16": torch.float16,
    "fp16": torch.float16,
    "half": torch.float16,
    "bfloat16": torch.bfloat16,
    "bf16": torch.bfloat16,
}


def resolve_dtype(name: str | torch.dtype) -> torch.dtype:
    """Map a dtype name (``fp32``, ``bfloat16``, ...) or a ``torch.dtype`` to a ``torch.dtype``."""
    if isinstance(name, torch.dtype):
        return name
    key = str(name).lower().replace("torch.", "")
    if key not in _DTYPE_NAMES:
        raise ConfigurationError(
            format_error(
                "config.resolve_dtype",
                "unknown dtype name",
                expected=sorted(_DTYPE_NAMES),
                observed=name,
                resolution="spell the dtype as one of the expected names",
            )
        )
    return _DTYPE_NAMES[key]


def _fail(where: str, problem: str, expected: Any, observed: Any, fix: str, cls: type = ConfigurationError) -> None:
    raise cls(format_error(where, problem, expected=expected, observed=observed, resolution=fix))


def _check(cond: bool, where: str, problem: str, expected: Any, observed: Any, fix: str, cls: type = ConfigurationError) -> None:
    if not cond:
        _fail(where, problem, expected, observed, fix, cls)


class SequenceParallelMode:
    """How the sequence dimension is split (string constants so YAML round-trips).

    ``tensor_group`` is Megatron sequence parallelism over the tensor group;
    ``independent`` gives the sequence its own grid dimension.
    """

    DISABLED = "disabled"
    TENSOR_GROUP = "tensor_group"
    INDEPENDENT = "independent"
    ALL = (DISABLED, TENSOR_GROUP, INDEPENDENT)


_DIM_FIELDS = ("data_parallel_size", "shard_parallel_size", "sequence_parallel_size", "tensor_parallel_size")


@dataclass(frozen=True)
class TopologyConfig:
    """Sizes of the four grid dimensions; their product is the world size."""

    data_parallel_size: int = 1
    shard_parallel_size: int = 1
    sequence_parallel_size: int = 1
    tensor_parallel_size: int = 1
    sequence_parallel_mode: str = SequenceParallelMode.DISABLED

    def __post_init__(self) -> None:
        where = "config.TopologyConfig"
        for name in _DIM_FIELDS:
            value = getattr(self, name)
            ok = isinstance(value, int) and not isinstance(value, bool) and value >= 1
            _check(ok, where, f"{name} has to be an integer of at least 1", ">= 1", value, f"set {name} to an integer of at least 1", TopologyError)
        mode = self.sequence_parallel_mode
        _check(mode in SequenceParallelMode.ALL, where, "sequence_parallel_mode is not a recognised value", list(SequenceParallelMode.ALL), mode,
               "pick a mode from the expected list", TopologyError)
        if mode != SequenceParallelMode.INDEPENDENT:
            _check(self.sequence_parallel_size == 1, where,
                   "sequence_parallel_size > 1 requires mode 'independent'; 'tensor_group' mode reuses the tensor ranks",
                   1, self.sequence_parallel_size,
                   "set sequence_parallel_mode='independent', or keep sequence_parallel_size=1", TopologyError)
        if mode == SequenceParallelMode.TENSOR_GROUP:
            _check(self.tensor_parallel_size > 1, where,
                   "sequence_parallel_mode='tensor_group' splits the sequence over the tensor group, which has one member",
                   "tensor_parallel_size > 1", self.tensor_parallel_size,
                   "sequence parallelism in tensor_group mode needs tensor_parallel_size above 1, or switch it off", TopologyError)

    @property
    def world_size(self) -> int:
        return math.prod(getattr(self, n) for n in _DIM_FIELDS)

    @property
    def effective_sequence_parallel_size(self) -> int:
        if self.sequence_parallel_mode == SequenceParallelMode.TENSOR_GROUP:
            return self.tensor_parallel_size
        if self.sequence_parallel_mode == SequenceParallelMode.INDEPENDENT:
            return self.sequence_parallel_size
        return 1

    @property
    def sequence_parallel_enabled(self) -> bool:
        return self.sequence_parallel_mode != SequenceParallelMode.DISABLED and self.effective_sequence_parallel_size > 1

    def validate_against_world_size(self, world_size: int) -> None:
        _check(
            self.world_size == world_size,
            "config.TopologyConfig.validate_against_world_size",
            f"parallel dimensions do not factor the world size (dp={self.data_parallel_size} x "
            f"shard={self.shard_parallel_size} x seq={self.sequence_parallel_size} x tensor={self.tensor_parallel_size})",
            world_size,
            self.world_size,
            "make the four sizes multiply to the number of launched processes",
            TopologyError,
        )

    @classmethod
    def for_world_size(cls, world_size: int, **overrides: Any) -> TopologyConfig:
        """Fill the first unspecified dimension so the product equals ``world_size``."""
        given = {k: v for k, v in overrides.items() if k in _DIM_FIELDS}
        missing = [d for d in _DIM_FIELDS if d not in given]
        product = math.prod(given.values()) if given else 1
        where = "config.TopologyConfig.for_world_size"
        _check(world_size % product == 0, where, "the supplied dimensions do not divide the world size",
               f"world_size divisible by {product}", world_size, "pick sizes whose product divides the world size", TopologyError)
        remainder = world_size // product
        resolved = dict(overrides)
        if remainder != 1:
            _check(bool(missing), where, "the four grid sizes multiply to fewer ranks than were launched",
                   world_size, product, "grow a grid dimension or start fewer ranks", TopologyError)
            resolved[missing[0]] = remainder
            missing = missing[1:]
        for name in missing:
            resolved.setdefault(name, 1)
        config = cls(**resolved)
        config.validate_against_world_size(world_size)
        return config


@dataclass(frozen=True)
class DDPConfig:
    """Bucketed data parallelism (reference ``config.py:361-418``)."""

    bucket_cap_mb: float = 25.0
    broadcast_buffers: bool = True
    find_unused_parameters: bool = False
    average_gradients: bool = True
    async_reduction: bool = True
    check_parameter_consistency: bool = True
    source_rank_in_group: int = 0
    fused_allreduce: bool = True

    def __post_init__(self) -> None:
        _check(self.bucket_cap_mb > 0, "config.DDPConfig", "the DDP bucket size (bucket_cap_mb) has to be greater than zero", "> 0", self.bucket_cap_mb,
               "set a bucket size in MiB above zero (25 is the usual choice)")
        _check(self.source_rank_in_group >= 0, "config.DDPConfig", "source_rank_in_group cannot be negative", ">= 0",
               self.source_rank_in_group, "give the index of the source within the data-parallel group")


@dataclass(frozen=True)
class FSDPConfig:
    """Flat-parameter sharding (reference ``config.py:421-491``)."""

    reshard_after_forward: bool = True
    average_gradients: bool = True
    auto_wrap_min_num_params: int = 0
    cpu_offload_params: bool = False
    limit_all_gather_bytes: int = 0
    check_reduction_order: bool = False
    use_padding: bool = True
    prefetch: bool = True
    fused_update: bool = True

    def __post_init__(self) -> None:
        _check(self.auto_wrap_min_num_params >= 0, "config.FSDPConfig", "auto_wrap_min_num_params cannot be negative",
               ">= 0", self.auto_wrap_min_num_params, "0 turns automatic unit wrapping off")
        _check(self.limit_all_gather_bytes >= 0, "config.FSDPConfig", "limit_all_gather_bytes cannot be negative",
               ">= 0", self.limit_all_gather_bytes, "0 turns the all-gather size limit off")
        _check(self.use_padding, "config.FSDPConfig",
               "use_padding=False is not supported: unpadded shards differ in size across ranks, which breaks the "
               "single-buffer all-gather / reduce-scatter", True, False, "leave use_padding at True")


@dataclass(frozen=True)
class TensorParallelConfig:
    """Tensor-parallel knobs (reference ``config.py:494-530``)."""

    gather_output: bool = False
    sequence_parallel: bool = False
    async_input_gradient_allreduce: bool = True
    init_method_std: float = 0.02
    fused_collectives: bool = True
    context_parallel_algorithm: str = "all_gather"

    def __post_init__(self) -> None:
        _check(self.init_method_std > 0, "config.TensorParallelConfig", "init_method_std has to be greater than zero", "> 0",
               self.init_method_std, "a standard deviation like 0.02 works for transformer weights")
        _check(self.context_parallel_algorithm in ("all_gather", "ring", "ulysses"), "config.TensorParallelConfig",
               "unknown context_parallel_algorithm (attention under sequence_parallel_mode='independent')",
               ["all_gather", "ring", "ulysses"], self.context_parallel_algorithm,
               "use 'all_gather' (fewer transfers), 'ring' (memory per rank independent of the sequence length) or "
               "'ulysses' (all-to-all to head groups; the flash kernel runs on the whole sequence)")


@dataclass(frozen=True)
class GradScalerConfig:
    """Dynamic loss scaling for fp16 (reference ``config.py:533-597``)."""

    enabled: bool = False
    init_scale: float = 65536.0
    growth_factor: float = 2.0
    backoff_factor: float = 0.5
    growth_interval: int = 2000
    max_scale: float = 2.0**24

    def __post_init__(self) -> None:
        where = "config.GradScalerConfig"
        _check(self.init_scale > 0, where, "the initial loss scale has to be greater than zero", "> 0", self.init_scale, "powers of two (65536 by default) keep the scaling exact")
        _check(self.growth_factor > 1.0, where, "the scale growth factor has to be above 1", "> 1.0", self.growth_factor, "use 2.0")
        _check(0.0 < self.backoff_factor < 1.0, where, "the scale backoff factor has to be strictly between 0 and 1", "0 < x < 1", self.backoff_factor, "use 0.5")
        _check(self.growth_interval >= 1, where, "growth_interval counts clean steps and has to be 1 or more", ">= 1", self.growth_interval, "use 2000")


@dataclass(frozen=True)
class MixedPrecisionConfig:
    """Compute / reduce / master dtypes (reference ``config.py:600-656``)."""

    enabled: bool = False
    param_dtype: str = "bfloat16"
    reduce_dtype: str = "float32"
    buffer_dtype: str = "float32"
    master_dtype: str = "float32"
    scaler: GradScalerConfig = field(default_factory=GradScalerConfig)

    def __post_init__(self) -> None:
        for name in ("param_dtype", "reduce_dtype", "buffer_dtype", "master_dtype"):
            resolve_dtype(getattr(self, name))
        if self.enabled and self.scaler.enabled:
            _check(resolve_dtype(self.param_dtype) is torch.float16, "config.MixedPrecisionConfig",
                   "loss scaling exists for float16 gradients, which underflow; bfloat16 and float32 do not need it", "scaler.enabled only together with param_dtype=float16",
                   self.param_dtype, "either compute in float16 or turn the scaler off")

    @property
    def compute_dtype(self) -> torch.dtype:
        return resolve_dtype(self.param_dtype) if self.enabled else resolve_dtype(self.master_dtype)

    @property
    def gradient_reduce_dtype(self) -> torch.dtype:
        return resolve_dtype(self.reduce_dtype) if self.enabled else resolve_dtype(self.master_dtype)


_ACTIVATIONS = ("gelu", "relu", "swiglu")


@dataclass(frozen=True)
class ModelConfig:
    """Model shape.  ``kind`` selects the MLP or the decoder transformer.

    The transformer covers both GPT-2 (``layernorm``, ``learned`` positions,
    ``gelu``, biases) and Llama (``rmsnorm``, ``rope``, ``swiglu``, no biases,
    ``num_kv_heads`` < ``num_heads`` for GQA).  See :meth:`gpt2_124m`,
    :meth:`llama_1b3` and :meth:`llama3_8b` for the benchmark shapes.
    """

    kind: str = "mlp"
    hidden_size: int = 64
    num_layers: int = 2
    input_size: int = 32
    output_size: int = 8
    vocab_size: int = 256
    num_heads: int = 4
    ffn_hidden_size: int = 0
    max_sequence_length: int = 64
    dropout: float = 0.0
    layer_norm_eps: float = 1e-5
    tie_word_embeddings: bool = False
    activation: str = "gelu"
    norm: str = "layernorm"
    position_embedding: str = "learned"
    rope_theta: float = 10000.0
    num_kv_heads: int = 0
    bias: bool = True
    fused_loss: bool = True
    init_std: float = 0.02

    def __post_init__(self) -> None:
        where = "config.ModelConfig"
        _check(self.kind in ("mlp", "transformer"), where, "unknown model kind", ["mlp", "transformer"], self.kind,
               "the model kinds are 'mlp' and 'transformer'")
        _check(self.activation in _ACTIVATIONS, where, "unknown activation", list(_ACTIVATIONS), self.activation,
               "use 'gelu', 'relu' or 'swiglu'")
        _check(self.norm in ("layernorm", "rmsnorm"), where, "unknown norm", ["layernorm", "rmsnorm"], self.norm,
               "use 'layernorm' or 'rmsnorm'")
        _check(self.position_embedding in ("learned", "rope"), where, "unknown position embedding", ["learned", "rope"],
               self.position_embedding, "use 'learned' or 'rope'")
        for name in ("hidden_size", "num_layers", "vocab_size", "num_heads", "max_sequence_length", "input_size", "output_size"):
            _check(getattr(self, name) >= 1, where, f"{name} must be positive", ">= 1", getattr(self, name),
                   f"set {name} to an integer of at least 1")
        if self.kind == "transformer":
            _check(self.hidden_size % self.num_heads == 0, where, "hidden_size has to split evenly into num_heads heads",
                   f"hidden_size % {self.num_heads} == 0", self.hidden_size, "pick a multiple of num_heads")
            _check(self.num_heads % self.resolved_num_kv_heads == 0, where, "num_heads must be a multiple of num_kv_heads",
                   f"num_heads % {self.resolved_num_kv_heads} == 0", self.num_heads, "pick num_kv_heads dividing num_heads")
        _check(0.0 <= self.dropout < 1.0, where, "dropout is a probability in [0, 1)", "0 <= p < 1", self.dropout, "use 0.0")
        _check(self.num_kv_heads >= 0, where, "num_kv_heads must be non-negative", ">= 0", self.num_kv_heads,
               "use 0 for multi-head attention")

    @property
    def resolved_ffn_hidden_size(self) -> int:
        return self.ffn_hidden_size if self.ffn_hidden_size > 0 else 4 * self.hidden_size

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def resolved_num_kv_heads(self) -> int:
        return self.num_kv_heads if self.num_kv_heads > 0 else self.num_heads

    @classmethod
    def gpt2_124m(cls, **overrides: Any) -> ModelConfig:
        """GPT-2 small: 12L, d768, 12 heads, V50257, S1024, tied embeddings."""
        base = dict(kind="transformer", hidden_size=768, num_layers=12, num_heads=12, vocab_size=50257,
                    max_sequence_length=1024, activation="gelu", norm="layernorm", position_embedding="learned",
                    tie_word_embeddings=True, bias=True)
        base.update(overrides)
        return cls(**base)

    @classmethod
    def llama_1b3(cls, **overrides: Any) -> ModelConfig:
        """Llama-style 1.3B: 24L, d2048, 16 heads, SwiGLU 5504, V32000, S2048."""
        base = dict(kind="transformer", hidden_size=2048, num_layers=24, num_heads=16, ffn_hidden_size=5504,
                    vocab_size=32000, max_sequence_length=2048, activation="swiglu", norm="rmsnorm",
                    position_embedding="rope", bias=False, layer_norm_eps=1e-5)
        base.update(overrides)
        return cls(**base)

    @classmethod
    def llama3_8b(cls, **overrides: Any) -> ModelConfig:
        """Llama-3-8B: 32L, d4096, 32q/8kv, ffn 14336, V128256, S4096, rope theta 5e5."""
        base = dict(kind="transformer", hidden_size=4096, num_layers=32, num_heads=32, num_kv_heads=8,
                    ffn_hidden_size=14336, vocab_size=128256, max_sequence_length=4096, activation="swiglu",
                    norm="rmsnorm", position_embedding="rope", rope_theta=500000.0, bias=False)
        base.update(overrides)
        return cls(**base)


@dataclass(frozen=True)
class DataConfig:
    """Synthetic dataset shape (reference ``config.py:773-819``)."""

    micro_batch_size: int = 4
    sequence_length: int = 16
    num_train_samples: int = 256
    num_eval_samples: int = 64
    seed: int = 1234
    shuffle: bool = True
    token_distribution: str = "recurrence"

    def __post_init__(self) -> None:
        for name in ("micro_batch_size", "sequence_length", "num_train_samples"):
            _check(getattr(self, name) >= 1, "config.DataConfig", f"{name} must be positive", ">= 1", getattr(self, name),
                   f"set {name} to an integer of at least 1")
        _check(self.num_eval_samples >= 0, "config.DataConfig", "num_eval_samples cannot be negative", ">= 0",
               self.num_eval_samples, "0 switches evaluation off")
        _check(self.token_distribution in ("recurrence", "uniform"), "config.DataConfig", "unknown token distribution",
               ["recurrence", "uniform"], self.token_distribution, "use 'recurrence' or 'uniform'")


@dataclass(frozen=True)
class OptimizerConfig:
    """AdamW or SGD (reference ``config.py:822-878``)."""

    name: str = "adamw"
    learning_rate: float = 1e-3
    weight_decay: float = 0.0
    betas: tuple[float, float] = (0.9, 0.999)
    eps: float = 1e-8
    momentum: float = 0.0
    cpu_offload_state: bool = False

    def __post_init__(self) -> None:
        where = "config.OptimizerConfig"
        _check(self.name in ("adamw", "sgd"), where, "unknown optimizer", ["adamw", "sgd"], self.name, "the optimizers available are 'adamw' and 'sgd'")
        _check(self.learning_rate > 0, where, "the learning rate has to be greater than zero", "> 0", self.learning_rate, "set learning_rate above zero")
        betas = tuple(self.betas)
        _check(len(betas) == 2 and all(0.0 <= b < 1.0 for b in betas), where, "betas has to be a pair of decay rates, each in [0, 1)",
               "two floats b1, b2 in [0, 1)", self.betas, "use (0.9, 0.999)")
        object.__setattr__(self, "betas", betas)


@dataclass(frozen=True)
class SchedulerConfig:
    """Learning-rate schedule (reference ``config.py:881-925``)."""

    name: str = "constant"
    warmup_steps: int = 0
    min_lr_ratio: float = 0.0

    def __post_init__(self) -> None:
        where = "config.SchedulerConfig"
        _check(self.name in ("constant", "linear", "cosine"), where, "unknown schedule", ["constant", "linear", "cosine"],
               self.name, "pick a schedule from the expected list")
        _check(self.warmup_steps >= 0, where, "warmup_steps cannot be negative", ">= 0", self.warmup_steps, "use 0")
        _check(0.0 <= self.min_lr_ratio <= 1.0, where, "min_lr_ratio is a fraction of the peak rate in [0, 1]", "0 <= r <= 1", self.min_lr_ratio, "use 0.0")


@dataclass(frozen=True)
class CheckpointConfig:
    """Checkpoint cadence and integrity checks (reference ``config.py:928-973``)."""

    directory: str = "checkpoints"
    save_every_steps: int = 0
    keep_last: int = 0
    save_optimizer_state: bool = True
    save_rng_state: bool = True
    verify_checksums_on_load: bool = True
    resume_from: str = ""

    def __post_init__(self) -> None:
        _check(self.save_every_steps >= 0, "config.CheckpointConfig", "save_every_steps cannot be negative", ">= 0",
               self.save_every_steps, "0 means no periodic saves")
        _check(self.keep_last >= 0, "config.CheckpointConfig", "keep_last cannot be negative", ">= 0", self.keep_last,
               "0 keeps all checkpoints")


@dataclass(frozen=True)
class TrainingConfig:
    """Loop control (reference ``config.py:976-1034``) plus ``cuda_graph``."""

    max_steps: int = 20
    gradient_accumulation_steps: int = 1
    max_grad_norm: float = 0.0
    seed: int = 0
    log_every_steps: int = 1
    eval_every_steps: int = 0
    deterministic: bool = True
    collect_metrics: bool = False
    cuda_graph: bool = False
    # Apply the optimizer update to each gradient bucket during the backward pass when the step
    # needs no global gradient quantity (no clipping, no norm metric, no loss scaling).  Off by
    # default: on GPT-2-124M it measured slower than one update after the backward (1 B200:
    # 11.63 vs 11.22 ms/step; 2 B200: 13.32 vs 13.10 ms/step), the update's memory traffic
    # competing with the backward's kernels.
    overlap_optimizer_step: bool = False

    def __post_init__(self) -> None:
        where = "config.TrainingConfig"
        _check(self.max_steps >= 0, where, "max_steps cannot be negative", ">= 0", self.max_steps, "give 0 or a larger number")
        _check(self.gradient_accumulation_steps >= 1, where, "gradient_accumulation_steps counts micro-batches and has to be 1 or more", ">= 1",
               self.gradient_accumulation_steps, "1 means one micro-batch per step (no accumulation)")
        _check(self.max_grad_norm >= 0, where, "max_grad_norm cannot be negative", ">= 0", self.max_grad_norm,
               "0 switches gradient clipping off")


@dataclass(frozen=True)
class ExperimentConfig:
    """Everything one run needs; YAML files map 1:1 onto it."""

    name: str = "experiment"
    backend: str = "auto"
    device: str = "auto"
    timeout_seconds: float = 300.0
    topology: TopologyConfig = field(default_factory=TopologyConfig)
    model: ModelConfig = field(default_factory=ModelConfig)
    data: DataConfig = field(default_factory=DataConfig)
    optimizer: OptimizerConfig = field(default_factory=OptimizerConfig)
    scheduler: SchedulerConfig = field(default_factory=SchedulerConfig)
    training: TrainingConfig = field(default_factory=TrainingConfig)
    checkpoint: CheckpointConfig = field(default_factory=CheckpointConfig)
    ddp: DDPConfig = field(default_factory=DDPConfig)
    fsdp: FSDPConfig = field(default_factory=FSDPConfig)
    tensor_parallel: TensorParallelConfig = field(default_factory=TensorParallelConfig)
    mixed_precision: MixedPrecisionConfig = field(default_factory=MixedPrecisionConfig)

    def __post_init__(self) -> None:
        where = "config.ExperimentConfig"
        _check(self.backend in ("auto", "gloo", "nccl"), where, "unknown backend", ["auto", "gloo", "nccl"], self.backend,
               "leave it at 'auto' to let the runtime pick the backend")
        _check(self.device in ("auto", "cpu", "cuda"), where, "unknown device", ["auto", "cpu", "cuda"], self.device,
               "leave it at 'auto' to let the runtime pick the device")
        _check(self.timeout_seconds > 0, where, "the collective timeout has to be greater than zero seconds", "> 0", self.timeout_seconds, "use e.g. 300")
        _check(not (self.backend == "gloo" and self.device == "cuda"), where,
               "Gloo on CUDA tensors supports only a few collectives and is never right for training",
               "backend='nccl' with device='cuda'", "backend='gloo', device='cuda'", "use nccl for CUDA or cpu for gloo")
        _check(not (self.tensor_parallel.sequence_parallel and not self.topology.sequence_parallel_enabled), where,
               "tensor_parallel.sequence_parallel is enabled but the topology has no sequence-parallel group",
               "topology.sequence_parallel_mode != 'disabled'", self.topology.sequence_parallel_mode,
               "set sequence_parallel_mode='tensor_group' with tensor_parallel_size > 1")

    def to_dict(self) -> dict[str, Any]:
        return dataclasses.asdict(self)

    def to_yaml(self, path: str | Path) -> Path:
        destination = Path(path)
        destination.parent.mkdir(parents=True, exist_ok=True)
        destination.write_text(yaml.safe_dump(self.to_dict(), sort_keys=False), encoding="utf-8")
        return destination

    @classmethod
    def from_dict(cls, payload: dict[str, Any]) -> ExperimentConfig:
        return _from_mapping(cls, payload, path="")


_T = TypeVar("_T")


def _from_mapping(cls: type[_T], payload: Any, *, path: str) -> _T:
    if not isinstance(payload, dict):
        _fail("config.from_dict", f"a YAML mapping was needed for {path or 'the top level'}", "mapping", type(payload).__name__,
              "the section is probably mis-indented in the YAML file")
    known = {f.name: f for f in fields(cls)}  # type: ignore[arg-type]
    unknown = sorted(set(payload) - set(known))
    if unknown:
        dotted = [f"{path}.{k}" if path else k for k in unknown]
        _fail("config.from_dict", f"key(s) not in the schema under {path or 'the top level'!r}", sorted(known), dotted,
              "delete or correct those keys: the loader refuses keys it does not know")
    kwargs = {name: _coerce(known[name].type, value, path=f"{path}.{name}" if path else name) for name, value in payload.items()}
    return cls(**kwargs)


def _coerce(field_type: Any, value: Any, *, path: str) -> Any:
    if isinstance(field_type, str):
        field_type = _NESTED.get(field_type, field_type)
    if isinstance(field_type, type) and is_dataclass(field_type):
        return _from_mapping(field_type, value, path=path)
    origin = get_origin(field_type)
    if origin is tuple and isinstance(value, (list, tuple)):
        return tuple(value)
    if origin is Union:
        args = [a for a in get_args(field_type) if a is not type(None)]
        if len(args) == 1 and value is not None:
            return _coerce(args[0], value, path=path)
    return value


_NESTED: dict[str, type] = {
    cls.__name__: cls
    for cls in (TopologyConfig, ModelConfig, DataConfig, OptimizerConfig, SchedulerConfig, TrainingConfig, CheckpointConfig,
                DDPConfig, FSDPConfig, TensorParallelConfig, MixedPrecisionConfig, GradScalerConfig)
}


def load_experiment_config(path: str | Path, **overrides: Any) -> ExperimentConfig:
    """Load a YAML experiment; keyword overrides are applied with ``dataclasses.replace``."""
    source = Path(path)
    if not source.is_file():
        _fail("config.load_experiment_config", "there is no configuration file at this path", "a path to a YAML file", str(source),
              "the shipped experiment files are in the configs/ directory")
    raw = yaml.safe_load(source.read_text(encoding="utf-8")) or {}
    config = ExperimentConfig.from_dict(raw)
    return dataclasses.replace(config, **overrides) if overrides else config
