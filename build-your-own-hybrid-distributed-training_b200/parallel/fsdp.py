"""Fully sharded data parallelism with flat parameters, plus hybrid sharding.

Each FSDP unit flattens its parameters (registration order), pads the flat
buffer to a multiple of the shard-group size and keeps only this rank's equal
shard as an ``nn.Parameter`` in the master dtype.  Forward all-gathers the
shard (cast to the compute dtype) into a full buffer whose views are bound to
the module attributes; with ``reshard_after_forward`` the buffer's storage is
freed after forward and refilled, *in the same tensor*, by a pre-backward hook
(the autograd version counter is preserved across the refill).  The
all-gather's adjoint reduce-scatters the full gradient (optionally followed by
an all-reduce over the replica group: HSDP), casts to the master dtype and
zeroes the padding.  ``no_sync`` accumulates unsharded gradients.  State dicts
use global coordinates, so checkpoints reshard across world sizes.

This follows ``src/hybrid_training/parallel/fsdp.py:150-1730`` (``FlatParamHandle``,
``_AllGatherFlatParam``, ``_PreBackwardUnshard``, auto-wrap, summon, state
dicts, ``optimizer_parameter_layout``).  Differences:

* parameters marked as sequence-parallel partial gradients are summed over
  the sequence-parallel group *before* the reduce-scatter (the reference
  reduces ``param.grad`` of the unwrapped model, which no longer holds them);
* ``prefetch=True`` issues the next unit's all-gather on a side stream while
  the current unit computes (the reference has no prefetch);
* on CUDA, with :meth:`FullyShardedDataParallel.enable_fused_update` (the
  engine calls it when the optimizer is ``FusedAdamW`` over the flat shards and
  the step needs no gradient norm), each unit's reduce-scatter, cast and
  sharded AdamW update run as ONE kernel over NVLink peer memory during the
  backward pass (``ops.comm.fsdp_reduce_scatter_adamw``), and the all-gathers
  read the peers' updated bf16 shards directly (``ops.comm.fsdp_all_gather``).
  The reference reduce-scatters with ``torch.distributed`` and steps
  ``torch.optim.AdamW`` afterwards (``fsdp.py:704-769``,
  ``sharded_optimizer.py:340-355``).
"""

from __future__ import annotations

import dataclasses
from collections.abc import Iterator, Sequence
from contextlib import contextmanager
from dataclasses import dataclass
from typing import Any

import torch
import torch.nn as nn

from ..config import FSDPConfig, MixedPrecisionConfig, resolve_dtype
from ..distributed.collectives import (
    CommunicationRecorder,
    ReduceOp,
    all_gather_object_in_group,
    all_gather_tensor,
    all_reduce,
    assert_metadata_consistent,
    broadcast,
    reduce_scatter_tensor,
    record_collective,
)
from ..distributed.groups import GroupHandle
from ..errors import ParameterConsistencyError, ShardingError, UnsupportedFeatureError, format_error
from ..logging import get_logger
from ..utils.tensors import FlatEntry, ShardRange, build_flat_layout, intersect_ranges
from ..utils.tracing import trace_range

__all__ = ["FlatParamHandle", "FullyShardedDataParallel", "PieceLayout", "ShardedTensorPiece", "reshard_state_dict_pieces"]

_LOG = get_logger(__name__)
_HAS_VERSION_GUARD = hasattr(torch.autograd, "_unsafe_preserve_version_counter")


@dataclass(frozen=True)
class ShardedTensorPiece:
    """A contiguous run ``[offset, offset + len)`` of a tensor's flattened global data."""

    name: str
    global_shape: tuple[int, ...]
    offset: int
    data: torch.Tensor

    @property
    def length(self) -> int:
        return int(self.data.numel())

    @property
    def range(self) -> ShardRange:
        return ShardRange(self.offset, self.length)


@dataclass(frozen=True)
class PieceLayout:
    """Where a piece of original tensor ``name`` sits inside a local flat shard."""

    name: str
    global_shape: tuple[int, ...]
    parameter_offset: int
    length: int
    local_offset: int


def _free_storage(t: torch.Tensor) -> None:
    storage = t.untyped_storage()
    if storage.size() > 0:
        storage.resize_(0)


def _alloc_storage(t: torch.Tensor, nbytes: int) -> None:
    storage = t.untyped_storage()
    if storage.size() != nbytes:
        storage.resize_(nbytes)


@contextmanager
def _keep_version(t: torch.Tensor) -> Iterator[None]:
    if _HAS_VERSION_GUARD:
        with torch.autograd._unsafe_preserve_version_counter(t):
            yield
    else:
        yield


class _AllGatherFlatParam(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, shard: torch.Tensor, handle: FlatParamHandle) -> torch.Tensor:
        ctx.handle = handle
        return handle.gather_full(shard)

    @staticmethod
    def backward(ctx: Any, grad_full: torch.Tensor) -> tuple[torch.Tensor | None, None]:
        return ctx.handle.reduce_scatter_gradient(grad_full), None


class _PreBackwardUnshard(torch.autograd.Function):
    """Identity on the unit's outputs whose backward refills the freed full buffer first."""

    @staticmethod
    def forward(ctx: Any, handle: FlatParamHandle, full: torch.Tensor, *tensors: torch.Tensor) -> Any:
        ctx.handle, ctx.full = handle, full
        outs = tuple(t.view_as(t) for t in tensors)
        return outs[0] if len(outs) == 1 else outs

    @staticmethod
    def backward(ctx: Any, *grads: torch.Tensor) -> tuple[Any, ...]:
        ctx.handle.refill(ctx.full)
        return (None, None, *grads)


class FlatParamHandle:
    """One FSDP unit's flat parameter: layout, shard, gather/reshard/refill and gradient reduction."""

    def __init__(self, named_parameters: Sequence[tuple[str, nn.Parameter]], locations: dict[int, list[tuple[nn.Module, str]]],
                 shard_group: GroupHandle, config: FSDPConfig, mixed_precision: MixedPrecisionConfig, device: torch.device, *,
                 replica_group: GroupHandle | None = None, recorder: CommunicationRecorder | None = None,
                 sequence_group: GroupHandle | None = None) -> None:
        rank = shard_group.global_rank
        if not named_parameters:
            raise ShardingError(format_error("fsdp.FlatParamHandle", "a sharding unit without parameters has nothing to shard", rank=rank,
                                             expected=">= 1", observed=0, resolution="only wrap modules that own parameters"))
        flags = {bool(p.requires_grad) for _, p in named_parameters}
        if len(flags) > 1:
            frozen = [n for n, p in named_parameters if not p.requires_grad]
            raise UnsupportedFeatureError(format_error(
                "fsdp.FlatParamHandle", "all parameters of a unit share one flat tensor and therefore one requires_grad flag",
                rank=rank, expected="all parameters of a unit trainable, or all frozen", observed=f"frozen: {frozen[:8]}",
                resolution="wrap the frozen submodule as its own unit, or unfreeze it"))
        self._shard_group, self._replica_group, self._sequence_group = shard_group, replica_group, sequence_group
        self._config, self._mixed_precision, self._device, self._recorder = config, mixed_precision, device, recorder
        self._requires_grad = flags.pop()
        self._names = tuple(n for n, _ in named_parameters)
        self._params = tuple(p for _, p in named_parameters)
        self._locations = {id(p): list(locations[id(p)]) for _, p in named_parameters}
        first = self._params[0].dtype
        mp = mixed_precision
        self._master_dtype = resolve_dtype(mp.master_dtype) if mp.enabled else first
        self._compute_dtype = resolve_dtype(mp.param_dtype) if mp.enabled else first
        self._reduce_dtype = resolve_dtype(mp.reduce_dtype) if mp.enabled else first
        self._entries, self._total_numel = build_flat_layout(list(named_parameters))
        g = shard_group.size
        self._shard_numel = -(-self._total_numel // g)
        self._padded_numel = self._shard_numel * g
        self._padding = self._padded_numel - self._total_numel
        if config.limit_all_gather_bytes:
            gathered = self._padded_numel * torch.empty(0, dtype=self._compute_dtype).element_size()
            if gathered > config.limit_all_gather_bytes:
                raise ShardingError(format_error(
                    "fsdp.FlatParamHandle", "gathering this unit needs more bytes than limit_all_gather_bytes allows", rank=rank,
                    expected=f"<= {config.limit_all_gather_bytes} bytes", observed=gathered,
                    resolution="lower auto_wrap_min_num_params to split the model into more units, or raise the limit"))
        self._sp_ranges = [(e.offset, e.numel) for e, p in zip(self._entries, self._params)
                           if getattr(p, "sequence_parallel_partial_grad", False)]
        self.flat_param = self._build_shard()
        self._attach_norm_weights()
        self._full: torch.Tensor | None = None
        self._full_bytes = 0
        self._is_sharded = True
        self._accumulator: torch.Tensor | None = None
        self._accumulate_only = False
        self._reduction_count = 0
        self._prefetched: tuple[torch.Tensor, torch.cuda.Event] | None = None
        # fused reduce-scatter + AdamW state (attach_fused_update): (workspace, optimizer, staging)
        self._fused: tuple[Any, Any, torch.Tensor] | None = None
        self._sym_shard: torch.Tensor | None = None
        self._gather_workspace: Any = None
        self._sym_stale = True
        self._detach_originals()

    # -- construction -----------------------------------------------------------------------------
    def _build_shard(self) -> nn.Parameter:
        flat = torch.zeros(self._padded_numel, dtype=self._master_dtype, device=self._device)
        for e, p in zip(self._entries, self._params):
            flat[e.offset:e.end].copy_(p.detach().to(device=self._device, dtype=self._master_dtype).reshape(-1))
        lo = self._shard_group.local_rank * self._shard_numel
        shard = flat[lo:lo + self._shard_numel].clone()
        if self._config.cpu_offload_params:
            shard = shard.cpu()
        return nn.Parameter(shard, requires_grad=self._requires_grad)

    def _attach_norm_weights(self) -> None:
        """Per-element multiplicity for the distributed gradient norm (shard width x TP width)."""
        full = torch.zeros(self._padded_numel, dtype=torch.float32)
        for e, p in zip(self._entries, self._params):
            factor = self._shard_group.size
            if not getattr(p, "is_tensor_parallel_replicated", True):
                factor *= int(getattr(p, "tensor_parallel_group_size", 1))
            full[e.offset:e.end] = float(factor)
        r = self.local_shard_range()
        self.flat_param.gradient_norm_scale_vector = full[r.start:r.end].clone()
        self.flat_param.gradient_norm_label = f"flat_param[{self._names[0]} .. {self._names[-1]}]"

    def _detach_originals(self) -> None:
        placeholder = torch.empty(0, dtype=self._compute_dtype, device=self._device)
        for p in self._params:
            for module, attr in self._locations[id(p)]:
                module._parameters.pop(attr, None)
                setattr(module, attr, placeholder)
            p.data = torch.empty(0, dtype=p.dtype, device=p.device)

    # -- properties ---------------------------------------------------------------------------------
    entries = property(lambda self: self._entries)
    managed_parameters = property(lambda self: self._params)
    names = property(lambda self: self._names)
    total_numel = property(lambda self: self._total_numel)
    padded_numel = property(lambda self: self._padded_numel)
    shard_numel = property(lambda self: self._shard_numel)
    padding = property(lambda self: self._padding)
    is_sharded = property(lambda self: self._is_sharded)
    shard_group = property(lambda self: self._shard_group)
    replica_group = property(lambda self: self._replica_group)
    compute_dtype = property(lambda self: self._compute_dtype)

    def local_shard_range(self) -> ShardRange:
        return ShardRange(self._shard_group.local_rank * self._shard_numel, self._shard_numel)

    # -- gather / reshard ----------------------------------------------------------------------------
    def _compute_shard(self, shard: torch.Tensor) -> torch.Tensor:
        s = shard if shard.device == self._device else shard.to(self._device, non_blocking=True)
        return s.to(self._compute_dtype).contiguous()

    def _all_gather_into(self, full: torch.Tensor, shard: torch.Tensor, *, background: bool = False) -> None:
        with trace_range(f"fsdp/all-gather {self._names[0]}"):
            self._all_gather_into_impl(full, shard, background=background)

    def _all_gather_into_impl(self, full: torch.Tensor, shard: torch.Tensor, *, background: bool) -> None:
        """Fill ``full`` with every rank's shard in the compute dtype (peer memory when fused, else NCCL).

        On the fused path a ``background`` gather (the prefetch, which overlaps the current unit's
        kernels) uses the copy engines; an on-demand gather uses the P2P load kernel.
        """
        if self._fused is not None:
            from ..ops.comm import fsdp_all_gather

            assert self._sym_shard is not None
            fsdp_all_gather(self._gather_workspace, self._sym_shard, full, copy_engine=background)
            record_collective(self._recorder, "fsdp_all_gather_p2p", self._shard_group.name,
                              num_bytes=full.numel() * full.element_size())
            return
        _, work = all_gather_tensor(self._compute_shard(shard), self._shard_group, out=full, recorder=self._recorder)
        work.wait()

    def prefetch(self) -> None:
        """Start this unit's all-gather on a side stream (consumed by the next ``gather_full``)."""
        if self._prefetched is not None or not self.flat_param.is_cuda or self._shard_group.is_trivial:
            return
        stream = _prefetch_stream(self._device)
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            full = torch.empty(self._padded_numel, dtype=self._compute_dtype, device=self._device)
            self._all_gather_into(full, self.flat_param.detach(), background=True)
            event = torch.cuda.Event()
            event.record(stream)
        full.record_stream(torch.cuda.current_stream())
        self._prefetched = (full, event)

    def gather_full(self, shard: torch.Tensor) -> torch.Tensor:
        if self._prefetched is not None:
            full, event = self._prefetched
            self._prefetched = None
            torch.cuda.current_stream().wait_event(event)
        else:
            full = torch.empty(self._padded_numel, dtype=self._compute_dtype, device=self._device)
            self._all_gather_into(full, shard)
        self._full = full
        self._full_bytes = full.untyped_storage().nbytes()
        self._is_sharded = False
        return full

    def bind_views(self, full: torch.Tensor) -> None:
        for e, p in zip(self._entries, self._params):
            view = full[e.offset:e.end].view(e.shape)
            for module, attr in self._locations[id(p)]:
                setattr(module, attr, view)

    def unbind_views(self) -> None:
        placeholder = torch.empty(0, dtype=self._compute_dtype, device=self._device)
        for p in self._params:
            for module, attr in self._locations[id(p)]:
                setattr(module, attr, placeholder)

    def unshard(self) -> torch.Tensor:
        full = _AllGatherFlatParam.apply(self.flat_param, self)
        self.bind_views(full)
        return full

    def reshard(self) -> None:
        if self._full is None or self._is_sharded:
            return
        if not _HAS_VERSION_GUARD:
            raise UnsupportedFeatureError(format_error(
                "fsdp.reshard", "this PyTorch lacks torch.autograd._unsafe_preserve_version_counter, needed to refill a "
                "freed flat parameter during backward", rank=self._shard_group.global_rank,
                resolution="use reshard_after_forward=False in the FSDP config"))
        _free_storage(self._full)
        self._is_sharded = True

    def refill(self, full: torch.Tensor) -> None:
        need = self._padded_numel * full.element_size()
        if full.untyped_storage().nbytes() == need:
            return
        with torch.no_grad(), _keep_version(full):
            _alloc_storage(full, need)
            self._all_gather_into(full.detach(), self.flat_param.detach())
        if full is self._full:
            self._is_sharded = False

    # -- fused reduce-scatter + AdamW ------------------------------------------------------------------------
    def fused_update_supported(self) -> bool:
        """Whether this unit can take the fused path (CUDA, bf16 compute, fp32 master, plain shard group)."""
        sp_partial = bool(self._sp_ranges) and self._sequence_group is not None and self._sequence_group.size > 1
        replicas = 1 if self._replica_group is None else self._replica_group.size
        return (self.flat_param.is_cuda and not self._shard_group.is_trivial and self._shard_group.size * replicas <= 8
                and not self._config.cpu_offload_params and self._compute_dtype == torch.bfloat16
                and self._master_dtype == torch.float32 and self._requires_grad and not sp_partial)

    def attach_fused_update(self, workspace: Any, optimizer: Any, staging: torch.Tensor, reduce_workspace: Any = None) -> None:
        """Route this unit's gradient through the fused kernel (collective: allocates a peer-mapped shard).

        ``workspace`` spans the shard group (the bf16 shards that the all-gathers read);
        ``reduce_workspace`` (hybrid sharding) spans the data-parallel x shard group and holds
        ``staging``, so one kernel sums every replica's gradient of this rank's slice.
        """
        self._sym_shard = workspace.allocate(self._shard_numel, torch.bfloat16)
        self._gather_workspace = workspace
        self._fused = (workspace if reduce_workspace is None else reduce_workspace, optimizer, staging)
        self._sym_stale = True

    def sync_fused_shard(self) -> None:
        """Write the bf16 copy of the fp32 master shard into the peer-mapped buffer (local; caller barriers)."""
        if self._sym_shard is not None:
            with torch.no_grad():
                self._sym_shard.copy_(self.flat_param.detach())
            self._sym_stale = False

    def mark_fused_shard_stale(self) -> None:
        """The fp32 master shard changed outside the fused kernel; refresh the bf16 copy before the next gather."""
        self._sym_stale = True

    fused = property(lambda self: self._fused is not None)
    fused_shard_stale = property(lambda self: self._fused is not None and self._sym_stale)

    def _fused_reduce_scatter_update(self, grad: torch.Tensor) -> None:
        from ..ops.comm import fsdp_reduce_scatter_adamw

        assert self._fused is not None and self._sym_shard is not None
        workspace, optimizer, staging = self._fused
        staging[:self._padded_numel].copy_(grad.reshape(-1))
        state = optimizer.state[self.flat_param]
        group = optimizer.param_groups[0]
        local = self.local_shard_range()
        valid = max(0, min(self._shard_numel, self._total_numel - local.start))
        summed = workspace.group.size  # shard ranks, times the replicas under hybrid sharding
        scale = 1.0 / summed if self._config.average_gradients else 1.0
        fsdp_reduce_scatter_adamw(workspace, staging, self._sym_shard, shard=self._shard_numel, valid=valid, scale=scale,
                                  param=self.flat_param.data, exp_avg=state["exp_avg"], exp_avg_sq=state["exp_avg_sq"],
                                  hyper=optimizer.hyper_parameters, betas=group["betas"], eps=group["eps"],
                                  weight_decay=group["weight_decay"], slice_index=self._shard_group.local_rank)
        record_collective(self._recorder, "fsdp_reduce_scatter_adamw", workspace.group.name,
                          num_bytes=self._padded_numel * staging.element_size())
        self._reduction_count += 1

    # -- gradient reduction --------------------------------------------------------------------------------
    def reduce_scatter_gradient(self, grad_full: torch.Tensor) -> torch.Tensor | None:
        with trace_range(f"fsdp/reduce-scatter {self._names[0]}"):
            return self._reduce_scatter_gradient(grad_full)

    def _reduce_scatter_gradient(self, grad_full: torch.Tensor) -> torch.Tensor | None:
        if self._fused is not None and not self._accumulate_only:
            # Fused path: the update happens here; autograd receives no shard gradient.
            grad = grad_full if self._accumulator is None else grad_full.to(self._reduce_dtype) + self._accumulator
            self._accumulator = None
            self._fused_reduce_scatter_update(grad)
            return None
        grad = grad_full.to(self._reduce_dtype).contiguous()
        if self._accumulate_only:
            self._accumulator = grad.clone() if self._accumulator is None else self._accumulator.add_(grad)
            return None
        if self._accumulator is not None:
            grad = grad + self._accumulator
            self._accumulator = None
        if self._sp_ranges and self._sequence_group is not None and self._sequence_group.size > 1:
            packed = torch.cat([grad[o:o + n] for o, n in self._sp_ranges])
            all_reduce(packed, self._sequence_group, op=ReduceOp.SUM, recorder=self._recorder).wait()
            cursor = 0
            for o, n in self._sp_ranges:
                grad[o:o + n].copy_(packed[cursor:cursor + n])
                cursor += n
        op = ReduceOp.AVG if self._config.average_gradients else ReduceOp.SUM
        shard_grad, work = reduce_scatter_tensor(grad, self._shard_group, op=op, recorder=self._recorder)
        work.wait()
        if self._replica_group is not None and self._replica_group.size > 1:
            all_reduce(shard_grad, self._replica_group, op=op, recorder=self._recorder).wait()
        self._reduction_count += 1
        shard_grad = shard_grad.to(self._master_dtype)
        if self._config.cpu_offload_params:
            shard_grad = shard_grad.cpu()
        self._zero_padding(shard_grad)
        return shard_grad

    def _zero_padding(self, shard_grad: torch.Tensor) -> None:
        if not self._padding:
            return
        local = self.local_shard_range()
        overlap = intersect_ranges(local, ShardRange(self._total_numel, self._padding))
        if overlap is not None:
            lo = overlap.start - local.start
            shard_grad[lo:lo + overlap.length].zero_()

    def free_full(self) -> None:
        if self._full is not None:
            _free_storage(self._full)
        self._full = None
        self._is_sharded = True
        self.unbind_views()

    def set_accumulate_without_reduction(self, value: bool) -> None:
        self._accumulate_only = value

    @property
    def has_pending_accumulation(self) -> bool:
        return self._accumulator is not None

    @property
    def reduction_count(self) -> int:
        return self._reduction_count

    # -- state in global coordinates -------------------------------------------------------------------------
    def local_piece_layout(self) -> list[PieceLayout]:
        local = self.local_shard_range()
        out = []
        for e in self._entries:
            overlap = intersect_ranges(local, ShardRange(e.offset, e.numel))
            if overlap is not None:
                out.append(PieceLayout(e.name, e.shape, overlap.start - e.offset, overlap.length, overlap.start - local.start))
        return out

    def local_pieces(self) -> list[ShardedTensorPiece]:
        shard = self.flat_param.detach()
        return [ShardedTensorPiece(p.name, p.global_shape, p.parameter_offset,
                                   shard[p.local_offset:p.local_offset + p.length].clone()) for p in self.local_piece_layout()]

    def load_local_pieces(self, pieces: dict[str, torch.Tensor]) -> None:
        local = self.local_shard_range()
        shard = self.flat_param.data
        for e in self._entries:
            t = pieces.get(e.name)
            if t is None:
                raise ShardingError(format_error("fsdp.load_local_pieces", "the state dict has no entry for a parameter",
                                                 rank=self._shard_group.global_rank, expected=e.name, observed=sorted(pieces)[:8],
                                                 resolution="load state saved from the same model"))
            if tuple(t.shape) != e.shape:
                raise ShardingError(format_error("fsdp.load_local_pieces", f"shape mismatch for {e.name!r}",
                                                 rank=self._shard_group.global_rank, expected=e.shape, observed=tuple(t.shape),
                                                 resolution="the state dict was written by a differently shaped model"))
            overlap = intersect_ranges(local, ShardRange(e.offset, e.numel))
            if overlap is None:
                continue
            dst = overlap.start - local.start
            src = overlap.start - e.offset
            shard[dst:dst + overlap.length].copy_(t.reshape(-1)[src:src + overlap.length].to(shard.dtype))
        self.mark_fused_shard_stale()

    def full_tensors(self) -> dict[str, torch.Tensor]:
        shard = self.flat_param.detach().to(self._device).contiguous()
        full, work = all_gather_tensor(shard, self._shard_group, recorder=self._recorder)
        work.wait()
        return {e.name: full[e.offset:e.end].view(e.shape).clone() for e in self._entries}

    def memory_summary(self) -> dict[str, int]:
        el = self.flat_param.element_size()
        grad = self.flat_param.grad
        return {"shard_bytes": self._shard_numel * el,
                "full_bytes": 0 if self._is_sharded or self._full is None else self._full_bytes,
                "grad_shard_bytes": 0 if grad is None else grad.numel() * grad.element_size(),
                "padding_bytes": self._padding * el}

    def metadata(self) -> dict[str, Any]:
        return {"names": list(self._names), "entries": [e.as_dict() for e in self._entries], "total_numel": self._total_numel,
                "padded_numel": self._padded_numel, "shard_numel": self._shard_numel}

    def __repr__(self) -> str:
        return (f"FlatParamHandle(params={len(self._params)}, total_numel={self._total_numel}, shard_numel={self._shard_numel}, "
                f"padding={self._padding}, sharded={self._is_sharded})")


_PREFETCH_STREAMS: dict[int, torch.cuda.Stream] = {}


def _prefetch_stream(device: torch.device) -> torch.cuda.Stream:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _PREFETCH_STREAMS:
        _PREFETCH_STREAMS[idx] = torch.cuda.Stream(device=device)
    return _PREFETCH_STREAMS[idx]


class FullyShardedDataParallel(nn.Module):
    """Shards ``module``'s parameters over ``shard_group`` (see the module docstring)."""

    def __init__(self, module: nn.Module, shard_group: GroupHandle, config: FSDPConfig | None = None, *,
                 replica_group: GroupHandle | None = None, mixed_precision: MixedPrecisionConfig | None = None,
                 device: torch.device | None = None, recorder: CommunicationRecorder | None = None,
                 sync_module_states: bool = True, sequence_group: GroupHandle | None = None) -> None:
        super().__init__()
        self._config = config or FSDPConfig()
        self._mixed_precision = mixed_precision or MixedPrecisionConfig()
        self._shard_group, self._replica_group, self._sequence_group = shard_group, replica_group, sequence_group
        self._recorder = recorder
        params = list(module.parameters())
        if not params:
            raise ShardingError(format_error("fsdp.__init__", "the wrapped module owns no parameters",
                                             rank=shard_group.global_rank, expected=">= 1", observed=0,
                                             resolution="shard a module that owns parameters"))
        self._device = device if device is not None else params[0].device
        if sync_module_states:
            for p in module.parameters():
                broadcast(p.data, shard_group, source_local_rank=0, recorder=recorder).wait()
            for b in module.buffers():
                if b.numel():
                    broadcast(b.data, shard_group, source_local_rank=0, recorder=recorder).wait()
        if self._config.auto_wrap_min_num_params > 0:
            module = self._auto_wrap(module)
        named, locations = _collect_managed_parameters(module)
        self.module = module
        self._handle: FlatParamHandle | None = None
        if named:
            self._handle = FlatParamHandle(named, locations, shard_group, self._config, self._mixed_precision, self._device,
                                           replica_group=replica_group, recorder=recorder, sequence_group=sequence_group)
            self.register_parameter("flat_param", self._handle.flat_param)
            assert_metadata_consistent(self._handle.metadata(), shard_group, name="the flat-parameter layout of every unit",
                                       operation="fsdp.verify_flat_layout")
        self._next_unit: FullyShardedDataParallel | None = None
        self._fused_units: list[FullyShardedDataParallel] | None = None  # set on the root by enable_fused_update
        self._check_no_cross_unit_tying()
        self._link_prefetch_order()

    def _auto_wrap(self, module: nn.Module) -> nn.Module:
        threshold = self._config.auto_wrap_min_num_params
        for name, child in list(module.named_children()):
            if isinstance(child, FullyShardedDataParallel):
                continue
            child = self._auto_wrap(child)
            managed, _ = _collect_managed_parameters(child)
            # Containers (ModuleList / ModuleDict) are iterated by their owners, so they are never
            # units themselves; their children are.
            container = isinstance(child, (nn.ModuleList, nn.ModuleDict))
            if not container and sum(p.numel() for _, p in managed) >= threshold:
                child = FullyShardedDataParallel(child, self._shard_group, dataclasses.replace(self._config, auto_wrap_min_num_params=0),
                                                 replica_group=self._replica_group, mixed_precision=self._mixed_precision,
                                                 device=self._device, recorder=self._recorder, sync_module_states=False,
                                                 sequence_group=self._sequence_group)
            setattr(module, name, child)
        return module

    def _link_prefetch_order(self) -> None:
        units = [u for u in self.fsdp_units() if u is not self and u._handle is not None]
        for a, b in zip(units, units[1:]):
            a._next_unit = b

    def _check_no_cross_unit_tying(self) -> None:
        seen: dict[int, str] = {}
        for unit in self.fsdp_units():
            if unit._handle is None:
                continue
            for name, p in zip(unit._handle.names, unit._handle.managed_parameters):
                prev = seen.get(id(p))
                if prev is not None and prev != name:
                    raise UnsupportedFeatureError(format_error(
                        "fsdp.check_tied_parameters", "a parameter is shared between two FSDP units; each would update its own "
                        "copy and the tie would break", rank=self._shard_group.global_rank,
                        expected="tied parameters inside one unit", observed=f"{prev!r} and {name!r} are the same tensor",
                        resolution="keep tied modules in one unit (raise auto_wrap_min_num_params) or untie them"))
                seen[id(p)] = name

    def __getattr__(self, name: str) -> Any:
        try:
            return super().__getattr__(name)
        except AttributeError:
            if name == "module":
                raise
            inner = self.__dict__.get("_modules", {}).get("module")
            if inner is None:
                raise
            return getattr(inner, name)

    # -- fused reduce-scatter + AdamW ------------------------------------------------------------------------
    def enable_fused_update(self, workspace: Any, optimizer: Any, *, accumulate: bool = False,
                            reduce_workspace: Any = None) -> bool:
        """Update every unit inside its gradient reduce-scatter kernel; returns whether the path is on.

        Requirements (decided from configuration only, so every rank decides alike): a peer-mapped
        ``workspace`` for the shard group, ``optimizer`` a CUDA ``FusedAdamW`` whose parameters are
        exactly the units' flat shards, bf16 compute with fp32 master shards, no CPU offload, at
        most 8 ranks summed.  With a replica group (hybrid sharding) ``reduce_workspace`` must span
        the data-parallel x shard group: the kernel then sums the gradients of every replica of
        the shard in the same pass (the reduce-scatter and the replica all-reduce in one).  The caller must not need the gradient afterwards (no clipping, no norm, no
        loss scaling): the optimizer step happens during the backward pass, unit by unit, and
        ``optimizer.step()`` must be skipped.  ``accumulate`` stages fp32 gradients (exact sums
        of accumulated micro-batches) instead of bf16 ones.  Collective over the shard group.
        """
        from ..optim.fused_adamw import FusedAdamW

        units = [u for u in self.fsdp_units() if u._handle is not None]
        if workspace is None or not units or not isinstance(optimizer, FusedAdamW) or not optimizer.flat_parameters.is_cuda:
            return False
        hybrid = self._replica_group is not None and self._replica_group.size > 1
        if hybrid and reduce_workspace is None:
            return False
        owned = {id(p) for p in optimizer.param_groups[0]["params"]}
        shards = {id(u._handle.flat_param) for u in units}
        if owned != shards or len(optimizer.param_groups) != 1:
            return False
        if not all(u._handle.fused_update_supported() for u in units):
            return False
        dtype = torch.float32 if accumulate else torch.bfloat16
        staging_ws = reduce_workspace if hybrid else workspace
        staging = staging_ws.allocate(max(u._handle.padded_numel for u in units), dtype)
        for u in units:
            u._handle.attach_fused_update(workspace, optimizer, staging, reduce_workspace if hybrid else None)
        self._fused_units = units
        self._fused_workspace = staging_ws
        _LOG.info("fsdp: fused reduce-scatter + AdamW over NVLink for %d units (%s gradient staging)", len(units),
                  str(dtype).replace("torch.", ""))
        return True

    @property
    def fused_update_enabled(self) -> bool:
        return self._fused_units is not None

    def sync_fused_shards(self) -> None:
        """Refresh stale peer-mapped bf16 shards from the fp32 masters, then barrier (collective).

        Called at the root's forward and by ``summon_full_params``: after a checkpoint load or any
        other write to the master shards through this API, every rank marks the same units stale,
        so every rank reaches the barrier.
        """
        if self._fused_units is None or not any(u._handle.fused_shard_stale for u in self._fused_units):
            return
        for u in self._fused_units:
            if u._handle.fused_shard_stale:
                u._handle.sync_fused_shard()
        # Stream-ordered barrier: a peer's all-gather launched after this reads the refreshed shards.
        all_reduce(torch.zeros(1, device=self._device), self._shard_group, op=ReduceOp.SUM, recorder=self._recorder).wait()

    def check_fused_status(self) -> None:
        """Raise if a fused kernel timed out waiting for a peer (reads a device word: host sync)."""
        if self._fused_units is not None:
            self._fused_workspace.check_status()

    def forward(self, *args: Any, **kwargs: Any) -> Any:
        if self._fused_units is not None:
            self.sync_fused_shards()
        full = self._handle.unshard() if self._handle is not None else None
        if self._config.prefetch and self._next_unit is not None and self._next_unit._handle is not None \
                and torch.is_grad_enabled():
            self._next_unit._handle.prefetch()
        out = self.module(*args, **kwargs)
        if self._handle is None:
            return out
        needs_backward = torch.is_grad_enabled() and self._handle.flat_param.requires_grad
        if self._config.reshard_after_forward:
            if needs_backward:
                out = _apply_pre_backward(self._handle, full, out)
            self._handle.reshard()
        elif not needs_backward:
            self._handle.reshard()
        return out

    @contextmanager
    def no_sync(self) -> Iterator[None]:
        units = [u for u in self.fsdp_units() if u._handle is not None]
        for u in units:
            u._handle.set_accumulate_without_reduction(True)
        try:
            yield
        finally:
            for u in units:
                u._handle.set_accumulate_without_reduction(False)

    def finish_backward(self) -> None:
        for u in self.fsdp_units():
            if u._handle is not None:
                u._handle.free_full()
        if self._config.check_reduction_order:
            order = [u._handle.reduction_count for u in self.fsdp_units() if u._handle is not None]
            gathered = all_gather_object_in_group(order, self._shard_group)
            if any(g != gathered[0] for g in gathered):
                raise ParameterConsistencyError(format_error(
                    "fsdp.finish_backward", "ranks ran a different number of gradient reduce-scatters for some "
                    "unit, so their collective sequences no longer match", rank=self._shard_group.global_rank, expected=gathered[0], observed=order,
                    resolution="every rank has to run the same modules in the same order"))

    def fsdp_units(self) -> list[FullyShardedDataParallel]:
        return [m for m in self.modules() if isinstance(m, FullyShardedDataParallel)]

    handle = property(lambda self: self._handle)
    config = property(lambda self: self._config)
    shard_group = property(lambda self: self._shard_group)

    @contextmanager
    def summon_full_params(self, *, writeback: bool = False) -> Iterator[None]:
        """Gather every unit's full parameters (bound as views); optionally write edits back to the shards."""
        units = [u for u in self.fsdp_units() if u._handle is not None]
        fulls = []
        self.sync_fused_shards()
        with torch.no_grad():
            for u in units:
                full = u._handle.gather_full(u._handle.flat_param.detach())
                u._handle.bind_views(full)
                fulls.append(full)
            try:
                yield
            finally:
                if writeback:
                    for u, full in zip(units, fulls):
                        r = u._handle.local_shard_range()
                        u._handle.flat_param.data.copy_(full[r.start:r.end].to(u._handle.flat_param.dtype))
                        u._handle.mark_fused_shard_stale()
                for u in units:
                    u._handle.free_full()

    def _units_with_prefix(self) -> list[tuple[FullyShardedDataParallel, str]]:
        out: list[tuple[FullyShardedDataParallel, str]] = [(self, "")]

        def walk(module: nn.Module, prefix: str) -> None:
            for name, child in module.named_children():
                p = f"{prefix}{name}."
                if isinstance(child, FullyShardedDataParallel):
                    out.append((child, p))
                    walk(child.module, p)
                else:
                    walk(child, p)

        walk(self.module, "")
        return out

    def sharded_state_dict(self) -> dict[str, ShardedTensorPiece]:
        out: dict[str, ShardedTensorPiece] = {}
        for unit, prefix in self._units_with_prefix():
            if unit._handle is None:
                continue
            for piece in unit._handle.local_pieces():
                out[prefix + piece.name] = ShardedTensorPiece(prefix + piece.name, piece.global_shape, piece.offset, piece.data)
        return out

    def full_state_dict(self) -> dict[str, torch.Tensor]:
        out: dict[str, torch.Tensor] = {}
        for unit, prefix in self._units_with_prefix():
            if unit._handle is not None:
                for name, t in unit._handle.full_tensors().items():
                    out[prefix + name] = t
        for name, b in self.original_named_buffers():
            out[name] = b.detach().clone()
        return out

    def load_full_state_dict(self, state_dict: dict[str, torch.Tensor]) -> None:
        for unit, prefix in self._units_with_prefix():
            if unit._handle is None:
                continue
            local = {n: state_dict[prefix + n] for n in unit._handle.names if prefix + n in state_dict}
            unit._handle.load_local_pieces(local)
        for name, b in self.original_named_buffers():
            if name in state_dict:
                b.data.copy_(state_dict[name].to(b.dtype))

    def optimizer_parameter_layout(self) -> list[tuple[nn.Parameter, list[PieceLayout]]]:
        prefixes = {id(u): p for u, p in self._units_with_prefix()}
        out = []
        for u in self.fsdp_units():
            if u._handle is None:
                continue
            prefix = prefixes[id(u)]
            out.append((u._handle.flat_param, [dataclasses.replace(i, name=prefix + i.name) for i in u._handle.local_piece_layout()]))
        return out

    def original_named_parameters(self) -> dict[str, tuple[tuple[int, ...], nn.Parameter]]:
        out = {}
        for unit, prefix in self._units_with_prefix():
            if unit._handle is not None:
                for e, p in zip(unit._handle.entries, unit._handle.managed_parameters):
                    out[prefix + e.name] = (e.shape, p)
        return out

    def original_named_buffers(self) -> list[tuple[str, torch.Tensor]]:
        found: list[tuple[str, torch.Tensor]] = []

        def walk(module: nn.Module, prefix: str) -> None:
            for name, b in module.named_buffers(recurse=False):
                if b is not None:
                    found.append((prefix + name, b))
            for name, child in module.named_children():
                walk(child.module if isinstance(child, FullyShardedDataParallel) else child, f"{prefix}{name}.")

        walk(self.module, "")
        return found

    def memory_summary(self) -> dict[str, int]:
        total = {"shard_bytes": 0, "full_bytes": 0, "grad_shard_bytes": 0, "padding_bytes": 0, "units": 0}
        for u in self.fsdp_units():
            if u._handle is not None:
                for k, v in u._handle.memory_summary().items():
                    total[k] += v
                total["units"] += 1
        return total

    def __repr__(self) -> str:
        return (f"FullyShardedDataParallel(shard_group={self._shard_group.name!r}, size={self._shard_group.size}, "
                f"units={len(self.fsdp_units())}, reshard_after_forward={self._config.reshard_after_forward})")


def _collect_managed_parameters(root: nn.Module) -> tuple[list[tuple[str, nn.Parameter]], dict[int, list[tuple[nn.Module, str]]]]:
    """Parameters owned directly by ``root`` (not by nested FSDP units), deduplicated, with every attribute location."""
    named: list[tuple[str, nn.Parameter]] = []
    where: dict[int, list[tuple[nn.Module, str]]] = {}

    def visit(module: nn.Module, prefix: str) -> None:
        for attr, p in list(module._parameters.items()):
            if p is None:
                continue
            if id(p) not in where:
                where[id(p)] = []
                named.append((prefix + attr, p))
            where[id(p)].append((module, attr))
        for name, child in module.named_children():
            if not isinstance(child, FullyShardedDataParallel):
                visit(child, f"{prefix}{name}.")

    visit(root, "")
    return named, where


def _apply_pre_backward(handle: FlatParamHandle, full: torch.Tensor, output: Any) -> Any:
    if isinstance(output, torch.Tensor):
        return _PreBackwardUnshard.apply(handle, full, output) if output.requires_grad else output
    if isinstance(output, dict):
        items = list(output.items())
    elif isinstance(output, (tuple, list)):
        items = list(enumerate(output))
    else:
        return output
    keys = [k for k, v in items if isinstance(v, torch.Tensor) and v.requires_grad]
    if not keys:
        return output
    mapping = dict(items)
    hooked = _PreBackwardUnshard.apply(handle, full, *(mapping[k] for k in keys))
    if isinstance(hooked, torch.Tensor):
        hooked = (hooked,)
    for k, v in zip(keys, hooked):
        mapping[k] = v
    if isinstance(output, dict):
        return type(output)(mapping)
    values = [mapping[k] for k, _ in items]
    return tuple(values) if isinstance(output, tuple) else values


def reshard_state_dict_pieces(pieces: Sequence[ShardedTensorPiece], global_shape: tuple[int, ...]) -> torch.Tensor:
    """Assemble a full tensor from flat pieces, requiring full coverage."""
    total = 1
    for d in global_shape:
        total *= d
    if not pieces:
        raise ShardingError(format_error("fsdp.reshard_state_dict_pieces", "no pieces supplied", expected=">= 1 piece",
                                         observed=0, resolution="the manifest should list shards for this tensor"))
    flat = torch.zeros(total, dtype=pieces[0].data.dtype)
    covered = torch.zeros(total, dtype=torch.bool)
    for piece in pieces:
        end = piece.offset + piece.length
        if end > total:
            raise ShardingError(format_error("fsdp.reshard_state_dict_pieces", f"piece for {piece.name!r} runs past the end",
                                             expected=f"offset + length <= {total}", observed=end,
                                             resolution="the saved layout does not fit this model"))
        flat[piece.offset:end] = piece.data.reshape(-1).to(flat.dtype)
        covered[piece.offset:end] = True
    if not bool(covered.all()):
        missing = int((~covered).sum())
        raise ShardingError(format_error("fsdp.reshard_state_dict_pieces", f"pieces leave {missing} element(s) uncovered",
                                         expected=f"{total} covered elements", observed=total - missing,
                                         resolution="a payload file is absent or lost entries"))
    return flat.view(global_shape)
