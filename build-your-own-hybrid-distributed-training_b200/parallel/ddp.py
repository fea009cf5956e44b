"""Bucketed data parallelism with gradient views and an in-kernel NVLink all-reduce.

Semantics kept from ``src/hybrid_training/parallel/ddp.py:266-837``:

* parameters are bucketed in **reverse registration order** (the order their
  gradients become ready), a new bucket starts at the byte cap or a
  dtype/device change;
* the (name, shape, dtype) list and the bucket layout are checked to be
  identical on every rank, and parameters/buffers are broadcast from the group
  source at construction;
* a bucket is reduced (``AVG`` = pre-divide + sum) as soon as all its
  gradients have arrived, but buckets are **launched strictly in index order**
  so every rank issues the same collective sequence; out-of-order readiness is
  counted;
* ``no_sync()`` accumulates without communication; ``find_unused_parameters``
  zero-fills the slots of parameters that got no gradient (otherwise that is
  an error, because the bucket could never complete);
* after synchronisation ``param.grad`` is a view into its bucket.

B200-native differences:

* all buckets are slices of **one flat fp32 gradient buffer**, and every
  parameter's ``main_grad`` is a view into it *from the first step*: the
  native wgrad GEMM writes gradients straight into the bucket (overwriting on
  the first micro-batch, accumulating after), so there is no copy into the
  bucket and no separate gradient tensor;
* on CUDA with a symmetric (peer-mapped) workspace for the group, the flat
  buffer lives in peer memory and each bucket is reduced by
  ``ops.comm.bucket_all_reduce`` -- a two-shot all-reduce that reads the peers'
  slices over NVLink, scales by ``1/G`` in the same pass and writes the result
  back to every rank -- issued on a communication stream that overlaps the
  rest of the backward pass; otherwise NCCL all-reduce (pre-multiplied sum)
  is used.
"""

from __future__ import annotations

from collections.abc import Iterator, Sequence
from contextlib import contextmanager
from dataclasses import dataclass
from typing import Any

import torch
import torch.nn as nn

from ..config import DDPConfig
from ..distributed.collectives import (
    AsyncWork,
    CommunicationRecorder,
    ReduceOp,
    all_reduce,
    assert_metadata_consistent,
    assert_tensor_consistent,
    broadcast,
    record_collective,
)
from ..distributed.groups import GroupHandle
from ..errors import ShardingError, format_error
from ..logging import get_logger
from ..utils.tracing import trace_range

__all__ = ["BucketLayout", "DDPStatistics", "DistributedDataParallel", "GradientBucket"]

_LOG = get_logger(__name__)
_MIB = 1 << 20
_ALIGN = 64  # elements: every bucket starts on a 256-byte boundary


@dataclass(frozen=True)
class BucketLayout:
    index: int
    parameter_names: tuple[str, ...]
    offsets: tuple[int, ...]
    numels: tuple[int, ...]
    total_numel: int
    dtype_str: str
    device_str: str

    def as_dict(self) -> dict[str, Any]:
        return {"index": self.index, "parameter_names": list(self.parameter_names), "offsets": list(self.offsets),
                "numels": list(self.numels), "total_numel": self.total_numel, "dtype": self.dtype_str}


class GradientBucket:
    """One contiguous slice of the flat gradient buffer and its readiness bookkeeping."""

    __slots__ = ("buffer", "launched", "layout", "parameters", "pending", "ready", "start", "work")

    def __init__(self, layout: BucketLayout, parameters: Sequence[nn.Parameter], buffer: torch.Tensor, start: int) -> None:
        self.layout = layout
        self.parameters = tuple(parameters)
        self.buffer = buffer
        self.start = start
        self.pending = len(parameters)
        self.ready = False
        self.launched = False
        self.work: AsyncWork | None = None

    @property
    def is_allocated(self) -> bool:
        return True

    def view_for(self, position: int) -> torch.Tensor:
        off, n = self.layout.offsets[position], self.layout.numels[position]
        return self.buffer[off:off + n].view(self.parameters[position].shape)

    def reset(self) -> None:
        self.pending = len(self.parameters)
        self.ready = self.launched = False
        self.work = None

    def num_bytes(self) -> int:
        return self.layout.total_numel * self.buffer.element_size()

    def __repr__(self) -> str:
        return f"GradientBucket(index={self.layout.index}, params={len(self.parameters)}, numel={self.layout.total_numel}, pending={self.pending})"


@dataclass
class DDPStatistics:
    steps: int = 0
    buckets_reduced: int = 0
    bytes_reduced: int = 0
    unused_parameters: tuple[str, ...] = ()
    out_of_order_buckets: int = 0

    def as_dict(self) -> dict[str, Any]:
        return {"steps": self.steps, "buckets_reduced": self.buckets_reduced, "bytes_reduced": self.bytes_reduced,
                "unused_parameters": list(self.unused_parameters), "out_of_order_buckets": self.out_of_order_buckets}


class _FusedLaunch:
    """Completion handle for an in-kernel bucket all-reduce issued on the comm stream."""

    def __init__(self, event: torch.cuda.Event, status: Any) -> None:
        self.event = event
        self.status = status

    def wait(self) -> None:
        torch.cuda.current_stream().wait_event(self.event)


class DistributedDataParallel(nn.Module):
    """Replicates ``module`` over ``group`` and averages gradients bucket by bucket."""

    def __init__(self, module: nn.Module, group: GroupHandle, config: DDPConfig | None = None, *,
                 recorder: CommunicationRecorder | None = None, workspace: Any = None) -> None:
        super().__init__()
        self.module = module
        self._group = group
        self._config = config or DDPConfig()
        self._recorder = recorder
        self._named_parameters: list[tuple[str, nn.Parameter]] = []
        seen: set[int] = set()
        for name, p in module.named_parameters():
            if p.requires_grad and id(p) not in seen:
                seen.add(id(p))
                self._named_parameters.append((name, p))
        if not self._named_parameters:
            raise ShardingError(format_error("ddp.__init__", "the module has no trainable parameters to synchronise",
                                             rank=group.global_rank, expected="one or more parameters that require gradients",
                                             observed=0, resolution="DDP only makes sense for a module with something to train"))
        self._name_of = {id(p): n for n, p in self._named_parameters}
        self._buckets: list[GradientBucket] = []
        self._bucket_of: dict[int, tuple[GradientBucket, int]] = {}
        self._handles: list[Any] = []
        self._require_backward_grad_sync = True
        self._backward_in_progress = False
        self._next_bucket = 0
        self._statistics = DDPStatistics()
        self._workspace = workspace if (self._config.fused_allreduce and not group.is_trivial) else None
        self._comm_stream: torch.cuda.Stream | None = None
        # Called as hook(start, numel) on the communication stream right after a bucket's all-reduce
        # was issued (flat-buffer coordinates): the optimizer updates the bucket during the backward.
        self.post_reduction_hook: Any = None
        self._draining = False  # True while finish_gradient_synchronization launches what is left
        if self._config.check_parameter_consistency:
            signature = [(n, tuple(p.shape), str(p.dtype)) for n, p in self._named_parameters]
            assert_metadata_consistent(signature, group, name="the names, shapes and dtypes of the trainable parameters",
                                       operation="ddp.verify_parameter_structure")
        self._broadcast_initial_state()
        self._build_buckets()
        self._register_hooks()
        _LOG.info("DDP ready over %r (size %d): %d parameters in %d buckets (%s all-reduce)", group.name, group.size,
                  len(self._named_parameters), len(self._buckets), "in-kernel" if self._workspace is not None else "NCCL")

    # -- construction -------------------------------------------------------------------------
    def _broadcast_initial_state(self) -> None:
        src = self._config.source_rank_in_group
        for _, p in self._named_parameters:
            broadcast(p.data, self._group, source_local_rank=src, recorder=self._recorder).wait()
        for _, b in self.module.named_buffers():
            if b is not None and b.numel():
                broadcast(b.data, self._group, source_local_rank=src, recorder=self._recorder).wait()

    def _build_buckets(self) -> None:
        cap = int(self._config.bucket_cap_mb * _MIB)
        groups: list[list[tuple[str, nn.Parameter]]] = []
        current: list[tuple[str, nn.Parameter]] = []
        size = 0
        key = None
        for name, p in reversed(self._named_parameters):
            k = (p.dtype, p.device)
            nbytes = p.numel() * p.element_size()
            if current and (k != key or size + nbytes > cap):
                groups.append(current)
                current, size = [], 0
            key = k
            current.append((name, p))
            size += nbytes
        if current:
            groups.append(current)
        # Gradients are reduced in fp32 (or the parameter dtype when wider).
        starts, total = [], 0
        for members in groups:
            starts.append(total)
            n = sum(p.numel() for _, p in members)
            total += -(-n // _ALIGN) * _ALIGN
        device = self._named_parameters[0][1].device
        grad_dtype = torch.float32 if self._named_parameters[0][1].dtype in (torch.float16, torch.bfloat16, torch.float32) else self._named_parameters[0][1].dtype
        if self._workspace is not None and device.type == "cuda":
            flat = self._workspace.allocate(total, grad_dtype)
        else:
            flat = torch.zeros(total, dtype=grad_dtype, device=device)
        self._flat_grad = flat
        for index, (members, start) in enumerate(zip(groups, starts)):
            offsets, numels, off = [], [], 0
            for _, p in members:
                offsets.append(off)
                numels.append(p.numel())
                off += p.numel()
            layout = BucketLayout(index, tuple(n for n, _ in members), tuple(offsets), tuple(numels), off,
                                  str(members[0][1].dtype), str(members[0][1].device))
            bucket = GradientBucket(layout, [p for _, p in members], flat[start:start + off], start)
            self._buckets.append(bucket)
            for pos, (_, p) in enumerate(members):
                self._bucket_of[id(p)] = (bucket, pos)
                p.main_grad = bucket.view_for(pos)
                p.main_grad_fresh = True
        if self._config.check_parameter_consistency:
            assert_metadata_consistent([b.layout.as_dict() for b in self._buckets], self._group,
                                       name="the bucket assignment of every gradient", operation="ddp.verify_bucket_layout")

    def _register_hooks(self) -> None:
        for _, p in self._named_parameters:
            p.grad_ready_hook = self._on_grad_ready
            self._handles.append(p.register_post_accumulate_grad_hook(self._on_autograd_grad))

    # -- backward-time bookkeeping ------------------------------------------------------------------
    def _on_autograd_grad(self, param: torch.Tensor) -> None:
        """Gradient produced by plain autograd (CPU ops, or ops without fused delivery)."""
        if param.grad is None:
            return
        from ..ops.grads import adopt_exposed_gradient, deliver_grad

        grad = param.grad
        adopt_exposed_gradient(param, from_autograd=True)
        param.grad = None
        deliver_grad(param, value=grad.detach().to(param.main_grad.dtype), native=False)

    def _on_grad_ready(self, param: torch.Tensor) -> None:
        if not self._require_backward_grad_sync:
            return
        self._backward_in_progress = True
        entry = self._bucket_of.get(id(param))
        if entry is None:
            return
        bucket, _ = entry
        if bucket.pending == 0:
            raise ShardingError(format_error(
                "ddp.on_grad_ready", "a gradient arrived for a bucket already reduced this iteration; backward() ran twice "
                "without a synchronisation boundary", rank=self._group.global_rank,
                expected="a single backward() between two synchronisations", observed=f"bucket {bucket.layout.index}",
                resolution="call finish_gradient_synchronization() after each backward(), or use no_sync()"))
        bucket.pending -= 1
        if bucket.pending == 0:
            bucket.ready = True
            if bucket.layout.index != self._next_bucket:
                self._statistics.out_of_order_buckets += 1
            if self._config.async_reduction:
                self._launch_ready_buckets()

    def _launch_ready_buckets(self) -> None:
        while self._next_bucket < len(self._buckets) and self._buckets[self._next_bucket].ready:
            self._launch(self._buckets[self._next_bucket])
            self._next_bucket += 1

    def _launch(self, bucket: GradientBucket) -> None:
        with trace_range(f"ddp/bucket {bucket.layout.index} all-reduce"):
            self._launch_bucket(bucket)

    def _launch_bucket(self, bucket: GradientBucket) -> None:
        average = self._config.average_gradients
        if self._workspace is not None and bucket.buffer.is_cuda:
            from ..ops.comm import bucket_all_reduce

            if self._comm_stream is None:
                # High priority: when compute kernels free SMs, the reduction's CTAs are scheduled
                # first, so the all-reduce keeps pace with the backward pass instead of trailing it.
                self._comm_stream = torch.cuda.Stream(device=bucket.buffer.device, priority=-1)
            self._comm_stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self._comm_stream):
                # Buckets reduced during the backward pass share the GPU with its GEMMs (narrow
                # kernel); the last bucket is reduced when the backward has finished (wide kernel).
                last = bucket.layout.index == len(self._buckets) - 1 or self._draining
                status = bucket_all_reduce(self._workspace, self._flat_grad, bucket.start, bucket.layout.total_numel,
                                           1.0 / self._group.size if average else 1.0, wide=last)
                if self.post_reduction_hook is not None:
                    self.post_reduction_hook(bucket.start, bucket.layout.total_numel)
                event = torch.cuda.Event()
                event.record(self._comm_stream)
            bucket.work = _FusedLaunch(event, status)  # type: ignore[assignment]
            record_collective(self._recorder, "all_reduce_nvlink", self._group.name, num_bytes=bucket.num_bytes())
        else:
            bucket.work = all_reduce(bucket.buffer, self._group, op=ReduceOp.AVG if average else ReduceOp.SUM,
                                     async_op=self._config.async_reduction, recorder=self._recorder)
            if self.post_reduction_hook is not None and bucket.buffer.is_cuda:
                if self._comm_stream is None:
                    self._comm_stream = torch.cuda.Stream(device=bucket.buffer.device, priority=-1)
                self._comm_stream.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(self._comm_stream):
                    bucket.work.wait()  # this stream waits for the reduction
                    self.post_reduction_hook(bucket.start, bucket.layout.total_numel)
                    event = torch.cuda.Event()
                    event.record(self._comm_stream)
                bucket.work = _FusedLaunch(event, None)  # type: ignore[assignment]
        bucket.launched = True
        self._statistics.buckets_reduced += 1
        self._statistics.bytes_reduced += bucket.num_bytes()

    def finish_gradient_synchronization(self, *, defer_last: bool = False) -> tuple[int, int, Any] | None:
        """Wait for every bucket and expose the averaged gradients as ``param.grad`` views.

        ``defer_last`` (in-kernel all-reduce only): leave the last bucket's reduction running and
        return ``(start, numel, wait)`` for it -- its range of the flat gradient buffer and a callable
        that makes the current stream wait for it -- so that work that does not read that range (the
        optimizer update of every other bucket) overlaps the last reduction.  ``None`` when nothing
        was deferred.
        """
        if not self._backward_in_progress:
            return None
        if not self._require_backward_grad_sync:
            self._backward_in_progress = False
            return None
        missing: list[str] = []
        for bucket in self._buckets:
            if bucket.pending == 0:
                continue
            for pos, p in enumerate(bucket.parameters):
                if getattr(p, "main_grad_fresh", False):
                    missing.append(self._name_of.get(id(p), f"<param#{pos}>"))
                    if self._config.find_unused_parameters:
                        bucket.view_for(pos).zero_()
                        p.main_grad_fresh = False
                        bucket.pending -= 1
            if bucket.pending == 0:
                bucket.ready = True
        if missing and not self._config.find_unused_parameters:
            raise ShardingError(format_error(
                "ddp.finish_gradient_synchronization", "parameters without a gradient leave their buckets incomplete, so those "
                "buckets would never be reduced", rank=self._group.global_rank,
                world_size=self._group.size, expected="a gradient for each trainable parameter",
                observed=f"no gradient for {len(missing)}, e.g. {missing[:8]}",
                resolution="set DDPConfig(find_unused_parameters=True), or stop marking unused parameters trainable"))
        self._statistics.unused_parameters = tuple(missing)
        self._draining = True
        try:
            self._launch_ready_buckets()
        finally:
            self._draining = False
        for bucket in self._buckets:
            if not bucket.launched:
                raise ShardingError(format_error("ddp.finish_gradient_synchronization",
                                                 f"bucket {bucket.layout.index} still waits for gradients after the backward pass", rank=self._group.global_rank,
                                                 expected="all buckets ready", observed=f"{bucket.pending} parameters pending",
                                                 resolution="the bucket counters are inconsistent (an internal error)"))
        deferred = None
        tail = self._buckets[-1] if self._buckets else None
        if (defer_last and tail is not None and isinstance(tail.work, _FusedLaunch)
                and all(p.dtype == tail.buffer.dtype for p in tail.parameters)):  # exposing a cast would read it
            deferred = (tail.start, tail.layout.total_numel, tail.work.wait)
        for bucket in self._buckets:
            if bucket.work is not None and not (deferred is not None and bucket is tail):
                bucket.work.wait()
        for bucket in self._buckets:
            for pos, p in enumerate(bucket.parameters):
                p.grad = bucket.view_for(pos).to(p.dtype) if p.dtype != bucket.buffer.dtype else bucket.view_for(pos)
                p._grad_exposed = True
            bucket.reset()
        self._next_bucket = 0
        self._backward_in_progress = False
        self._statistics.steps += 1
        return deferred

    def check_collective_status(self) -> None:
        """Raise :class:`KernelError` if an in-kernel bucket all-reduce gave up waiting for a peer.

        Reads the workspace's device status word (a host synchronisation).  The training engine
        reads it together with the step's loss; code that drives this module directly calls it
        after the steps it wants checked.
        """
        if self._workspace is not None:
            self._workspace.check_status()

    # -- forward / context managers ----------------------------------------------------------------
    def forward(self, *args: Any, **kwargs: Any) -> Any:
        if self._backward_in_progress and self._require_backward_grad_sync:
            raise ShardingError(format_error(
                "ddp.forward", "the last backward pass was never synchronised, so its gradients are "
                "still per-rank", rank=self._group.global_rank,
                expected="finish_gradient_synchronization() to close each backward()", observed="buckets still waiting for their reduction",
                resolution="call finish_gradient_synchronization() before the next forward"))
        if self._config.broadcast_buffers and self.training:
            src = self._config.source_rank_in_group
            for _, b in self.module.named_buffers():
                if b.numel():
                    broadcast(b.data, self._group, source_local_rank=src, recorder=self._recorder).wait()
        return self.module(*args, **kwargs)

    @contextmanager
    def no_sync(self) -> Iterator[None]:
        previous = self._require_backward_grad_sync
        self._require_backward_grad_sync = False
        try:
            yield
        finally:
            self._require_backward_grad_sync = previous

    # -- introspection / teardown ------------------------------------------------------------------
    @property
    def group(self) -> GroupHandle:
        return self._group

    @property
    def config(self) -> DDPConfig:
        return self._config

    @property
    def statistics(self) -> DDPStatistics:
        return self._statistics

    @property
    def communication_stream(self) -> torch.cuda.Stream | None:
        """The stream bucket reductions (and their post-reduction hooks) are issued on, once created."""
        return self._comm_stream

    @property
    def flat_gradient_buffer(self) -> torch.Tensor:
        return self._flat_grad

    def bucket_layouts(self) -> tuple[BucketLayout, ...]:
        return tuple(b.layout for b in self._buckets)

    @property
    def reduction_path(self) -> str:
        """``"in-kernel"`` when buckets are reduced by the symmetric-memory kernel, else ``"process-group"``."""
        return "in-kernel" if self._workspace is not None else "process-group"

    def communication_summary(self) -> str:
        if self._recorder is None:
            return "no recorder attached: construct with recorder=CommunicationRecorder() to count collectives"
        return self._recorder.summary()

    def parameters_and_names(self) -> tuple[tuple[str, nn.Parameter], ...]:
        return tuple(self._named_parameters)

    def verify_replica_consistency(self, *, atol: float = 0.0) -> None:
        for name, p in self._named_parameters:
            assert_tensor_consistent(p.data, self._group, name=f"parameter {name!r}", atol=atol,
                                     operation="ddp.verify_replica_consistency")

    def drain_pending_reductions(self) -> int:
        """Wait for in-flight reductions and reset bookkeeping (safe teardown after an exception)."""
        drained = 0
        for bucket in self._buckets:
            if bucket.work is not None:
                bucket.work.wait()
                drained += 1
            bucket.reset()
        self._next_bucket = 0
        self._backward_in_progress = False
        return drained

    def teardown(self) -> None:
        self.drain_pending_reductions()
        for h in self._handles:
            h.remove()
        self._handles.clear()
        for _, p in self._named_parameters:
            for attr in ("grad_ready_hook", "main_grad"):
                if hasattr(p, attr):
                    delattr(p, attr)
        self._bucket_of.clear()
        self._buckets.clear()

    def __repr__(self) -> str:
        return (f"DistributedDataParallel(group={self._group.name!r}, size={self._group.size}, buckets={len(self._buckets)}, "
                f"params={len(self._named_parameters)})")
