"""Tensor-parallel layers: column-, row-, QKV- and vocab-parallel.

Semantics follow ``src/hybrid_training/parallel/tensor_parallel.py:157-854``:

* **initialisation** draws the *full* matrix under a derived seed and keeps
  this rank's slice, so every tensor-parallel width initialises the same
  global model (and a width-1 layer equals ``nn.Linear`` built with the same
  seed, see :func:`hybrid_training.models.build_reference_linear`);
* **column-parallel**: entry is ``copy_to_group`` (or the sequence-parallel
  all-gather), output stays feature-sharded unless ``gather_output``;
* **row-parallel**: the partial product is all-reduced (or reduce-scattered
  along the sequence under SP) and the bias is added *after* the reduction;
  under SP the bias gradient is a partial sum, marked for the SP all-reduce;
* **vocab-parallel embedding**: out-of-shard ids give zero rows, then an
  all-reduce (or a sequence reduce-scatter when the model runs SP);
* partition markers (``tensor_parallel_partition_dim`` etc.) drive the
  distributed gradient norm and the checkpoint's ``#tpKofN`` keys.

What is new: :class:`QKVParallelLinear` fuses the q/k/v projections into one
column-parallel GEMM (one sequence all-gather per attention instead of the
reference's three) with an *interleaved-by-partition* global layout
``[q_0 k_0 v_0 | q_1 k_1 v_1 | ...]`` and supports grouped-query attention; all
matrix products go through :func:`hybrid_training.ops.linear` (tcgen05 GEMM
with fused bias/GELU epilogues on CUDA); and when the group has a symmetric
workspace the SP all-gather / reduce-scatter run inside the GEMM
(:mod:`hybrid_training.ops.comm`).
"""

from __future__ import annotations

import math
from typing import Any

import torch
import torch.nn as nn

from .. import ops
from ..autograd.collectives import (
    all_gather_along_dim,
    copy_to_group,
    gather_from_group,
    gather_from_sequence_parallel_region,
    reduce_from_group,
    reduce_scatter_to_group,
    scatter_to_group,
)
from ..distributed.collectives import ReduceOp, all_reduce
from ..distributed.groups import GroupHandle
from ..errors import TensorParallelError, format_error
from ..utils.reproducibility import derive_seed, temporary_seed
from ..utils.tensors import split_tensor_along_dim

__all__ = [
    "ColumnParallelLinear",
    "QKVParallelLinear",
    "RowParallelLinear",
    "TensorParallelFeedForward",
    "TensorParallelMLPBlock",
    "VocabParallelEmbedding",
    "VocabParallelHead",
    "all_reduce_sequence_parallel_gradients",
    "init_linear_parameters",
    "mark_sequence_parallel_partial",
]

SEQUENCE_DIM = 1


def init_linear_parameters(weight: torch.Tensor, bias: torch.Tensor | None, *, in_features: int) -> None:
    """``nn.Linear``'s default init (Kaiming-uniform weight, fan-in uniform bias)."""
    nn.init.kaiming_uniform_(weight, a=math.sqrt(5))
    if bias is not None:
        bound = 1.0 / math.sqrt(in_features) if in_features > 0 else 0.0
        nn.init.uniform_(bias, -bound, bound)


def _divide(value: int, parts: int, *, what: str, group: GroupHandle) -> int:
    if value % parts:
        raise TensorParallelError(format_error(
            "tensor_parallel.validate_divisible",
            f"{what} must be divisible by the tensor-parallel size; uneven splits give ranks different shapes",
            rank=group.global_rank, expected=f"{what} % {parts} == 0", observed=f"{what}={value}, remainder={value % parts}",
            resolution=f"choose {what} as a multiple of {parts}, or use fewer tensor-parallel ranks"))
    return value // parts


def _factory(device: torch.device | None, dtype: torch.dtype | None) -> dict[str, Any]:
    out: dict[str, Any] = {}
    if device is not None:
        out["device"] = device
    if dtype is not None:
        out["dtype"] = dtype
    return out


def _full_linear_init(out_features: int, in_features: int, bias: bool, seed: int, factory: dict[str, Any],
                      std: float | None = None) -> tuple[torch.Tensor, torch.Tensor | None]:
    with temporary_seed(derive_seed(seed, "tensor-parallel-init")):
        weight = torch.empty(out_features, in_features, **factory)
        b = torch.empty(out_features, **factory) if bias else None
        if std is None:
            init_linear_parameters(weight, b, in_features=in_features)
        else:
            nn.init.normal_(weight, mean=0.0, std=std)
            if b is not None:
                nn.init.zeros_(b)
    return weight, b


def _mark_partitioned(param: nn.Parameter, group: GroupHandle, *, partition_dim: int) -> None:
    param.tensor_parallel_partition_dim = partition_dim
    param.tensor_parallel_group_name = group.name
    param.tensor_parallel_group_size = group.size
    param.is_tensor_parallel_replicated = False


def _mark_replicated(param: nn.Parameter, group: GroupHandle) -> None:
    param.tensor_parallel_partition_dim = None
    param.tensor_parallel_group_name = group.name
    param.tensor_parallel_group_size = group.size
    param.is_tensor_parallel_replicated = True


def mark_sequence_parallel_partial(param: nn.Parameter) -> None:
    """Flag a replicated parameter whose gradient is a per-rank partial sum under SP."""
    param.sequence_parallel_partial_grad = True


def _fused_comm(group: GroupHandle, x: torch.Tensor) -> Any:
    """The symmetric workspace for in-kernel SP collectives, or ``None`` for the NCCL path."""
    if group.is_trivial or not x.is_cuda:
        return None
    from ..distributed.context import current_context, is_context_active

    from ..ops.comm import HAS_FUSED_TENSOR_PARALLEL

    if not HAS_FUSED_TENSOR_PARALLEL or not is_context_active() or not getattr(current_context(), "fused_tensor_collectives", False):
        return None
    return current_context().symmetric_workspace(group.name)


class ColumnParallelLinear(nn.Module):
    """``Y = X A^T + b`` with ``A`` split along its output features."""

    def __init__(self, in_features: int, out_features: int, group: GroupHandle, *, bias: bool = True,
                 gather_output: bool = False, sequence_parallel: bool = False, init_seed: int = 0,
                 device: torch.device | None = None, dtype: torch.dtype | None = None,
                 activation: str | None = None, init_std: float | None = None) -> None:
        super().__init__()
        if sequence_parallel and gather_output:
            raise TensorParallelError(format_error(
                "tensor_parallel.ColumnParallelLinear", "sequence_parallel keeps the output feature-sharded for a row layer; "
                "gathering it too would undo both savings", rank=group.global_rank,
                expected="an ungathered output under sequence parallelism", observed="both True", resolution="leave gather_output off"))
        self.in_features, self.out_features, self.group = in_features, out_features, group
        self.gather_output, self.sequence_parallel, self.activation = gather_output, sequence_parallel, activation
        self.output_features_per_partition = _divide(out_features, group.size, what="out_features", group=group)
        full_w, full_b = _full_linear_init(out_features, in_features, bias, init_seed, _factory(device, dtype), init_std)
        self.weight = nn.Parameter(split_tensor_along_dim(full_w, 0, group.size)[group.local_rank].clone())
        if full_b is not None:
            self.bias: nn.Parameter | None = nn.Parameter(split_tensor_along_dim(full_b, 0, group.size)[group.local_rank].clone())
        else:
            self.register_parameter("bias", None)
        _mark_partitioned(self.weight, group, partition_dim=0)
        if self.bias is not None:
            _mark_partitioned(self.bias, group, partition_dim=0)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.sequence_parallel:
            workspace = _fused_comm(self.group, x)
            if workspace is not None:
                from ..ops.comm import all_gather_linear

                out = all_gather_linear(x, self.weight, self.bias, workspace, self.group, activation=self.activation, owner=id(self))
                if out is not None:
                    return out
            x = gather_from_sequence_parallel_region(x, self.group, dim=SEQUENCE_DIM)
        else:
            workspace = _fused_comm(self.group, x)
            if workspace is not None:
                from ..ops.comm import column_linear_reduced_grad

                out = column_linear_reduced_grad(x, self.weight, self.bias, workspace, self.group, activation=self.activation,
                                                 owner=id(self))
                if out is not None:
                    return gather_from_group(out, self.group, dim=-1) if self.gather_output else out
            x = copy_to_group(x, self.group)
        out = ops.linear(x, self.weight, self.bias, activation=self.activation)
        if self.gather_output:
            out = gather_from_group(out, self.group, dim=-1)
        return out

    def full_weight(self) -> torch.Tensor:
        return all_gather_along_dim(self.weight.detach(), self.group, 0)

    def full_bias(self) -> torch.Tensor | None:
        return None if self.bias is None else all_gather_along_dim(self.bias.detach(), self.group, 0)

    def load_from_linear(self, linear: nn.Linear) -> None:
        _check_shape(self, linear)
        with torch.no_grad():
            self.weight.copy_(split_tensor_along_dim(linear.weight.detach(), 0, self.group.size)[self.group.local_rank])
            if self.bias is not None:
                _require_bias(self, linear)
                self.bias.copy_(split_tensor_along_dim(linear.bias.detach(), 0, self.group.size)[self.group.local_rank])

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"per_partition={self.output_features_per_partition}, tp_size={self.group.size}, bias={self.bias is not None}, "
                f"gather_output={self.gather_output}, sequence_parallel={self.sequence_parallel}")


def _check_shape(layer: nn.Module, linear: nn.Linear) -> None:
    if tuple(linear.weight.shape) != (layer.out_features, layer.in_features):
        raise TensorParallelError(format_error("tensor_parallel.load_from_linear", "the weight has another shape",
                                               rank=layer.group.global_rank, expected=(layer.out_features, layer.in_features),
                                               observed=tuple(linear.weight.shape), resolution="the dense layer has other feature sizes"))


def _require_bias(layer: nn.Module, linear: nn.Linear) -> None:
    if linear.bias is None:
        raise TensorParallelError(format_error("tensor_parallel.load_from_linear", "this layer has a bias but the reference does not",
                                               rank=layer.group.global_rank, expected="a bias tensor", observed=None,
                                               resolution="build the parallel layer without a bias"))


class RowParallelLinear(nn.Module):
    """``Y = X A^T + b`` with ``A`` split along its input features; ``b`` is added after the reduction."""

    def __init__(self, in_features: int, out_features: int, group: GroupHandle, *, bias: bool = True,
                 input_is_parallel: bool = True, sequence_parallel: bool = False, init_seed: int = 0,
                 device: torch.device | None = None, dtype: torch.dtype | None = None, init_std: float | None = None) -> None:
        super().__init__()
        self.in_features, self.out_features, self.group = in_features, out_features, group
        self.input_is_parallel, self.sequence_parallel = input_is_parallel, sequence_parallel
        self.input_features_per_partition = _divide(in_features, group.size, what="in_features", group=group)
        full_w, full_b = _full_linear_init(out_features, in_features, bias, init_seed, _factory(device, dtype), init_std)
        self.weight = nn.Parameter(split_tensor_along_dim(full_w, 1, group.size)[group.local_rank].clone())
        if full_b is not None:
            self.bias: nn.Parameter | None = nn.Parameter(full_b.clone())
        else:
            self.register_parameter("bias", None)
        _mark_partitioned(self.weight, group, partition_dim=1)
        if self.bias is not None:
            _mark_replicated(self.bias, group)
            if sequence_parallel:
                mark_sequence_parallel_partial(self.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.input_is_parallel:
            x = scatter_to_group(x, self.group, dim=-1)
        # A width-1 group adds the bias inside the GEMM epilogue; otherwise after the reduction.
        fused_bias = self.bias if self.group.is_trivial else None
        if self.sequence_parallel:
            workspace = _fused_comm(self.group, x)
            if workspace is not None:
                from ..ops.comm import linear_reduce_scatter

                out = linear_reduce_scatter(x, self.weight, workspace, self.group, owner=id(self))
                if out is not None:
                    return out if self.bias is None else out + self.bias.to(out.dtype)
        if not self.sequence_parallel:
            workspace = _fused_comm(self.group, x)
            if workspace is not None:
                from ..ops.comm import linear_all_reduce

                out = linear_all_reduce(x, self.weight, workspace, self.group, owner=id(self))
                if out is not None:
                    return out if self.bias is None else out + self.bias.to(out.dtype)
        partial = ops.linear(x, self.weight, fused_bias)
        if self.group.is_trivial:
            return partial
        out = reduce_scatter_to_group(partial, self.group, SEQUENCE_DIM) if self.sequence_parallel else reduce_from_group(partial, self.group)
        return out if self.bias is None else out + self.bias.to(out.dtype)

    def full_weight(self) -> torch.Tensor:
        return all_gather_along_dim(self.weight.detach(), self.group, 1)

    def load_from_linear(self, linear: nn.Linear) -> None:
        _check_shape(self, linear)
        with torch.no_grad():
            self.weight.copy_(split_tensor_along_dim(linear.weight.detach(), 1, self.group.size)[self.group.local_rank])
            if self.bias is not None:
                _require_bias(self, linear)
                self.bias.copy_(linear.bias.detach())

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"per_partition={self.input_features_per_partition}, tp_size={self.group.size}, bias={self.bias is not None}, "
                f"input_is_parallel={self.input_is_parallel}, sequence_parallel={self.sequence_parallel}")


class QKVParallelLinear(ColumnParallelLinear):
    """Fused q/k/v projection, column-parallel by heads, GQA-aware.

    Rank ``r`` holds ``[q heads of r; k heads of r; v heads of r]``; the global
    weight is the rank-major interleave of those slices.  Each of q, k and v is
    initialised as its own full matrix (seed streams ``attn-q``/``attn-k``/
    ``attn-v``) before slicing, matching three separate column layers.
    """

    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int, head_dim: int, group: GroupHandle, *,
                 bias: bool = True, sequence_parallel: bool = False, init_seed: int = 0,
                 device: torch.device | None = None, dtype: torch.dtype | None = None, init_std: float | None = None) -> None:
        nn.Module.__init__(self)
        t = group.size
        _divide(num_heads, t, what="num_heads", group=group)
        _divide(num_kv_heads, t, what="num_kv_heads", group=group)
        self.in_features = hidden_size
        self.out_features = (num_heads + 2 * num_kv_heads) * head_dim
        self.group, self.gather_output, self.sequence_parallel, self.activation = group, False, sequence_parallel, None
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.output_features_per_partition = self.out_features // t
        factory = _factory(device, dtype)
        w_parts, b_parts = [], []
        for name, heads in (("attn-q", num_heads), ("attn-k", num_kv_heads), ("attn-v", num_kv_heads)):
            w, b = _full_linear_init(heads * head_dim, hidden_size, bias, derive_seed(init_seed, name), factory, init_std)
            w_parts.append(split_tensor_along_dim(w, 0, t)[group.local_rank])
            if b is not None:
                b_parts.append(split_tensor_along_dim(b, 0, t)[group.local_rank])
        self.weight = nn.Parameter(torch.cat(w_parts, 0).contiguous())
        if bias:
            self.bias = nn.Parameter(torch.cat(b_parts, 0).contiguous())
        else:
            self.register_parameter("bias", None)
        _mark_partitioned(self.weight, group, partition_dim=0)
        if self.bias is not None:
            _mark_partitioned(self.bias, group, partition_dim=0)

    def canonical(self, gathered: torch.Tensor) -> torch.Tensor:
        """Reorder a rank-major gathered tensor ``[q_0 k_0 v_0 | q_1 ...]`` (dim 0) into ``[q; k; v]``."""
        t = self.group.size
        q, kv = self.num_heads * self.head_dim // t, self.num_kv_heads * self.head_dim // t
        parts = [p.split([q, kv, kv], dim=0) for p in gathered.chunk(t, dim=0)]
        return torch.cat([p[0] for p in parts] + [p[1] for p in parts] + [p[2] for p in parts], dim=0)

    def full_weight(self) -> torch.Tensor:
        """The full ``[(H + 2 Hkv) * D, hidden]`` projection in the canonical ``[q; k; v]`` order."""
        return self.canonical(all_gather_along_dim(self.weight.detach(), self.group, 0))

    def extra_repr(self) -> str:
        return (f"hidden={self.in_features}, heads={self.num_heads}, kv_heads={self.num_kv_heads}, head_dim={self.head_dim}, "
                f"tp_size={self.group.size}, bias={self.bias is not None}, sequence_parallel={self.sequence_parallel}")


class VocabParallelEmbedding(nn.Module):
    """Embedding table split along the vocabulary; out-of-shard rows are zero, then reduced."""

    def __init__(self, num_embeddings: int, embedding_dim: int, group: GroupHandle, *, init_seed: int = 0,
                 init_std: float = 0.02, device: torch.device | None = None, dtype: torch.dtype | None = None) -> None:
        super().__init__()
        self.num_embeddings, self.embedding_dim, self.group = num_embeddings, embedding_dim, group
        self.embeddings_per_partition = _divide(num_embeddings, group.size, what="num_embeddings", group=group)
        self.vocab_start = group.local_rank * self.embeddings_per_partition
        self.vocab_end = self.vocab_start + self.embeddings_per_partition
        with temporary_seed(derive_seed(init_seed, "tensor-parallel-init")):
            full = torch.empty(num_embeddings, embedding_dim, **_factory(device, dtype))
            nn.init.normal_(full, mean=0.0, std=init_std)
        self.weight = nn.Parameter(split_tensor_along_dim(full, 0, group.size)[group.local_rank].clone())
        _mark_partitioned(self.weight, group, partition_dim=0)

    def local_lookup(self, token_ids: torch.Tensor, positions: torch.Tensor | None = None) -> torch.Tensor:
        """This shard's contribution (zeros for foreign ids), before any reduction."""
        return ops.embedding(token_ids, self.weight, positions, vocab_start=self.vocab_start)

    def forward(self, token_ids: torch.Tensor, positions: torch.Tensor | None = None, *, reduce: bool = True) -> torch.Tensor:
        """Embedded tokens (fp32 on CUDA).  ``positions`` (rows ``[:S]`` added) is only allowed at width 1,
        where it fuses the position add into the gather; ``reduce=False`` returns this shard's partial sum."""
        if positions is not None and self.group.size > 1:
            raise TensorParallelError(format_error("tensor_parallel.VocabParallelEmbedding", "positions can only be fused at width 1",
                                                   rank=self.group.global_rank, expected=1, observed=self.group.size,
                                                   resolution="add the position rows after the reduction"))
        out = self.local_lookup(token_ids, positions)
        return out if (self.group.size == 1 or not reduce) else reduce_from_group(out, self.group)

    def full_weight(self) -> torch.Tensor:
        return all_gather_along_dim(self.weight.detach(), self.group, 0)

    def extra_repr(self) -> str:
        return (f"num_embeddings={self.num_embeddings}, embedding_dim={self.embedding_dim}, "
                f"per_partition={self.embeddings_per_partition}, tp_size={self.group.size}")


def _activation_fn(name: str):
    from ..models.mlp import build_activation

    return build_activation(name)


class TensorParallelFeedForward(nn.Module):
    """``fc2(act(fc1(x)))`` with fc1 column-parallel and fc2 row-parallel.

    ``activation='swiglu'`` makes fc1 produce ``[gate; up]`` per rank (width
    ``2 * ffn / T``) and applies ``silu(gate) * up``.  GELU is fused into the
    fc1 GEMM epilogue; with a width-1 tensor group both activations, and their
    gradients, run inside the two GEMMs' epilogues.
    """

    def __init__(self, hidden_size: int, ffn_hidden_size: int, group: GroupHandle, *, activation: str = "gelu",
                 bias: bool = True, sequence_parallel: bool = False, init_seed: int = 0,
                 device: torch.device | None = None, dtype: torch.dtype | None = None, init_std: float | None = None,
                 output_init_std: float | None = None) -> None:
        super().__init__()
        self.activation_name = activation
        swiglu = activation == "swiglu"
        self.fc1: nn.Module
        if swiglu:
            self.fc1 = _GateUpParallelLinear(hidden_size, ffn_hidden_size, group, bias=bias, sequence_parallel=sequence_parallel,
                                             init_seed=derive_seed(init_seed, "ffn-fc1"), device=device, dtype=dtype,
                                             init_std=init_std)
        else:
            self.fc1 = ColumnParallelLinear(hidden_size, ffn_hidden_size, group, bias=bias, gather_output=False,
                                            sequence_parallel=sequence_parallel, init_seed=derive_seed(init_seed, "ffn-fc1"),
                                            device=device, dtype=dtype, activation="gelu" if activation == "gelu" else None,
                                            init_std=init_std)
        self.fc2 = RowParallelLinear(ffn_hidden_size, hidden_size, group, bias=bias, input_is_parallel=True,
                                     sequence_parallel=sequence_parallel, init_seed=derive_seed(init_seed, "ffn-fc2"),
                                     device=device, dtype=dtype, init_std=output_init_std)
        self._activation = None if activation in ("gelu", "swiglu") else _activation_fn(activation)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # The fused paths read fc1's and fc2's weights directly instead of calling them, so they are
        # taken only when both are the plain layers: a layer wrapped as its own FSDP unit gathers its
        # parameters when it is called, and holds a placeholder until then.
        plain = type(self.fc1) in (ColumnParallelLinear, _GateUpParallelLinear) and type(self.fc2) is RowParallelLinear
        if plain and self.activation_name == "gelu" and self.fc1.group.is_trivial and x.is_cuda:
            # Width-1 group: both linears and the GELU as one fused op (GELU' in fc2's dgrad epilogue).
            return ops.gelu_mlp(x, self.fc1.weight, self.fc1.bias, self.fc2.weight, self.fc2.bias)
        if (plain and self.activation_name == "swiglu" and self.fc1.group.is_trivial and x.is_cuda
                and ops.swiglu_mlp_supported(self.fc1.output_features_per_partition // 2)):
            # Width-1 group: SwiGLU in fc1's epilogue (gate and up rows in one tile) and its
            # gradient in fc2's data-gradient epilogue.
            return ops.swiglu_mlp(x, self.fc1.weight, self.fc1.bias, self.fc2.weight, self.fc2.bias)
        h = self.fc1(x)
        if self.activation_name == "swiglu":
            h = ops.swiglu(h)
        elif self._activation is not None:
            h = self._activation(h)
        return self.fc2(h)


class _GateUpParallelLinear(ColumnParallelLinear):
    """SwiGLU input projection: rank ``r`` holds ``[gate_r; up_r]`` (gate and up each split by features)."""

    def __init__(self, hidden_size: int, ffn_hidden_size: int, group: GroupHandle, *, bias: bool, sequence_parallel: bool,
                 init_seed: int, device: torch.device | None, dtype: torch.dtype | None, init_std: float | None) -> None:
        nn.Module.__init__(self)
        t = group.size
        _divide(ffn_hidden_size, t, what="ffn_hidden_size", group=group)
        self.in_features, self.out_features = hidden_size, 2 * ffn_hidden_size
        self.group, self.gather_output, self.sequence_parallel, self.activation = group, False, sequence_parallel, None
        self.output_features_per_partition = self.out_features // t
        factory = _factory(device, dtype)
        ws, bs = [], []
        for name in ("gate", "up"):
            w, b = _full_linear_init(ffn_hidden_size, hidden_size, bias, derive_seed(init_seed, name), factory, init_std)
            ws.append(split_tensor_along_dim(w, 0, t)[group.local_rank])
            if b is not None:
                bs.append(split_tensor_along_dim(b, 0, t)[group.local_rank])
        self.weight = nn.Parameter(torch.cat(ws, 0).contiguous())
        if bias:
            self.bias = nn.Parameter(torch.cat(bs, 0).contiguous())
        else:
            self.register_parameter("bias", None)
        _mark_partitioned(self.weight, group, partition_dim=0)
        if self.bias is not None:
            _mark_partitioned(self.bias, group, partition_dim=0)


class TensorParallelMLPBlock(nn.Module):
    """``act(column_linear(x))`` with the output gathered (used by the TP MLP model)."""

    def __init__(self, in_features: int, out_features: int, group: GroupHandle, *, activation: str = "gelu",
                 bias: bool = True, init_seed: int = 0, device: torch.device | None = None, dtype: torch.dtype | None = None) -> None:
        super().__init__()
        self.linear = ColumnParallelLinear(in_features, out_features, group, bias=bias, gather_output=True,
                                           init_seed=init_seed, device=device, dtype=dtype)
        self.activation_name = activation
        self._activation = _activation_fn(activation)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._activation(self.linear(x))


def all_reduce_sequence_parallel_gradients(module: nn.Module, group: GroupHandle, *, recorder: Any = None) -> int:
    """Sum the partial gradients of parameters marked ``sequence_parallel_partial_grad`` over ``group``.

    All partial gradients are packed into one flat buffer and reduced with a
    single collective (the reference issues one per parameter).
    """
    if group.size == 1:
        return 0
    targets = []
    for p in module.parameters():
        if not getattr(p, "sequence_parallel_partial_grad", False):
            continue
        g = getattr(p, "main_grad", None)
        g = p.grad if g is None or p.grad is not None else g
        if g is not None:
            targets.append(g)
    if not targets:
        return 0
    flat = torch.cat([g.detach().reshape(-1).float() for g in targets])
    all_reduce(flat, group, op=ReduceOp.SUM, recorder=recorder).wait()
    offset = 0
    for g in targets:
        n = g.numel()
        g.detach().copy_(flat[offset:offset + n].view(g.shape))
        offset += n
    return len(targets)


class VocabParallelHead(ColumnParallelLinear):
    """Output projection split by vocabulary rows; with ``targets`` it returns the fused mean cross-entropy.

    Without targets it is the reference's column-parallel head (full logits via
    ``gather_output``).  With targets the logits never leave the rank: the head GEMM
    feeds :func:`hybrid_training.ops.lm_head_cross_entropy`, which exchanges three
    floats per token over the tensor group.  The input must already carry the
    adjoint that sums the per-rank partial input gradients (``copy_to_group`` or the
    sequence-parallel gather), which the model inserts.
    """

    def forward(self, x: torch.Tensor, targets: torch.Tensor | None = None) -> torch.Tensor:
        if targets is None:
            return super().forward(x)
        group = self.group if self.group.size > 1 else None
        start = self.group.local_rank * self.output_features_per_partition
        return ops.lm_head_cross_entropy(x, self.weight, targets, group=group, vocab_start=start, vocab_size=self.out_features)
