"""AdamW applied during the backward pass, one gradient group at a time.

In the reference the optimizer step starts after the whole backward pass and every gradient
reduction have finished (``src/hybrid_training/training/engine.py:388-398``).  When the step needs
nothing global from the gradients -- no clipping, no gradient-norm metric, no loss scaling -- each
parameter's update depends only on its own gradient, so it can run as soon as that gradient is
final.  :class:`OverlappedAdamW` does that for :class:`~hybrid_training.optim.fused_adamw.FusedAdamW`:

* with data parallelism, DDP calls :meth:`bucket_reduced` right after it issued a bucket's
  all-reduce on its communication stream; the AdamW kernel for the bucket's slice of the flat
  buffers is queued on that stream behind the reduction;
* without it, this class tracks the parameters itself in groups of about ``group_bytes`` (in the
  order their gradients become ready, the reverse of registration) and queues each group's update
  on a side stream as soon as the group's last gradient has been written.

The update kernel is the flat AdamW of ``csrc/optim.cu`` in its small-footprint form: one
128-thread block per SM, which fits beside the persistent GEMM that the backward pass runs at the
same time.  A group is updated only after every backward op that reads its weights has been
issued: the native linear layers compute the input gradient (the GEMM that reads the weight)
before they deliver the weight gradient, and the side stream waits for everything issued on the
compute stream up to the delivery.  :meth:`finish` joins the side stream into the compute stream,
so the next forward pass reads updated weights.
"""

from __future__ import annotations

from collections.abc import Iterator
from contextlib import contextmanager
from typing import Any

import torch

from .. import ops
from .fused_adamw import FusedAdamW

__all__ = ["OverlappedAdamW"]

_ALIGN = 64  # elements: the flat buffers' per-tensor alignment


class OverlappedAdamW:
    """Runs a :class:`FusedAdamW` step in slices during the backward pass (see the module docstring)."""

    def __init__(self, optimizer: FusedAdamW, *, group_bytes: int = 25 << 20, track_parameters: bool = True) -> None:
        self.optimizer = optimizer
        self._stream: torch.cuda.Stream | None = None
        self._armed = False
        self._pending_autograd: list[torch.nn.Parameter] = []
        self._handles: list[Any] = []
        self._groups: list[tuple[int, int, list[torch.nn.Parameter]]] = []
        self._remaining: list[int] = []
        self._group_of: dict[int, int] = {}
        self._launched: list[bool] = []
        self._external = not track_parameters
        if track_parameters:
            self._build_groups(group_bytes)

    # -- grouping (no data parallelism) ---------------------------------------------------------------------
    def _build_groups(self, group_bytes: int) -> None:
        opt = self.optimizer
        order = sorted(zip(opt._offsets, opt._params), key=lambda t: t[0], reverse=True)
        current: list[tuple[int, torch.nn.Parameter]] = []
        size = 0
        for off, p in order:
            nbytes = p.numel() * 4
            if current and size + nbytes > group_bytes:
                self._add_group(current)
                current, size = [], 0
            current.append((off, p))
            size += nbytes
        if current:
            self._add_group(current)
        for index, (_, _, members) in enumerate(self._groups):
            for p in members:
                self._group_of[id(p)] = index
                p.grad_ready_hook = self._on_ready
                self._handles.append(p.register_post_accumulate_grad_hook(self._on_autograd_grad))
        self._remaining = [len(m) for _, _, m in self._groups]
        self._launched = [False] * len(self._groups)

    def _add_group(self, members: list[tuple[int, torch.nn.Parameter]]) -> None:
        start = min(off for off, _ in members)
        end = max(off + -(-p.numel() // _ALIGN) * _ALIGN for off, p in members)
        self._groups.append((start, end - start, [p for _, p in members]))

    # -- step protocol -------------------------------------------------------------------------------------------------
    def begin(self) -> None:
        """Before the forward pass: stage this step's hyper-parameters on the compute stream."""
        self.optimizer.stage_hyper_parameters()

    @contextmanager
    def armed(self) -> Iterator[None]:
        """Updates fire only while armed: around the backward pass of the step's last micro-batch."""
        self._armed = True
        try:
            yield
        finally:
            self._armed = False

    def _side_stream(self) -> torch.cuda.Stream:
        if self._stream is None:
            self._stream = torch.cuda.Stream(device=self.optimizer.flat_parameters.device, priority=-1)
        return self._stream

    def _launch(self, start: int, numel: int) -> None:
        opt = self.optimizer
        group = opt.param_groups[0]
        beta1, beta2 = group["betas"]
        end = start + numel
        copy = opt._compute_flat[start:end] if opt._compute_flat is not None else None
        ops.adamw_flat(opt._param_flat[start:end], opt._grad_flat[start:end], opt._exp_avg[start:end],
                       opt._exp_avg_sq[start:end], copy, opt.hyper_parameters, beta1=beta1, beta2=beta2, eps=group["eps"],
                       weight_decay=group["weight_decay"], resident=True)

    def bucket_reduced(self, start: int, numel: int) -> None:
        """DDP hook: called on DDP's communication stream right after a bucket's all-reduce was issued."""
        padded = -(-numel // _ALIGN) * _ALIGN
        self._launch(start, min(padded, self.optimizer.flat_parameters.numel() - start))

    def _on_autograd_grad(self, param: torch.Tensor) -> None:
        if param.grad is None or not self._armed:
            return
        from ..ops.grads import adopt_exposed_gradient, deliver_grad

        grad = param.grad
        adopt_exposed_gradient(param, from_autograd=True)
        param.grad = None
        deliver_grad(param, value=grad.detach().to(param.main_grad.dtype), native=False)

    def _on_ready(self, param: torch.Tensor) -> None:
        if not self._armed:
            return
        index = self._group_of.get(id(param))
        if index is None or self._launched[index]:
            return
        self._remaining[index] -= 1
        if self._remaining[index] == 0:
            self._fire(index)

    def _fire(self, index: int) -> None:
        start, numel, _ = self._groups[index]
        side = self._side_stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self._launch(start, numel)
        self._launched[index] = True

    def finish(self, comm_stream: torch.cuda.Stream | None = None) -> None:
        """After the backward pass: update what never became ready, then join the update stream(s)."""
        if not self._external:
            for index, (_, _, members) in enumerate(self._groups):
                if not self._launched[index]:
                    for p in members:  # parameters without a gradient this step take a zero gradient
                        if getattr(p, "main_grad_fresh", False):
                            p.main_grad.zero_()
                            p.main_grad_fresh = False
                    self._fire(index)
            self._remaining = [len(m) for _, _, m in self._groups]
            self._launched = [False] * len(self._groups)
        current = torch.cuda.current_stream()
        if self._stream is not None:
            current.wait_stream(self._stream)
        if comm_stream is not None:
            current.wait_stream(comm_stream)
        for p in self.optimizer._params:
            p.compute_copy_version = p._version

    def close(self) -> None:
        for h in self._handles:
            h.remove()
        self._handles.clear()
        for _, _, members in self._groups:
            for p in members:
                if getattr(p, "grad_ready_hook", None) == self._on_ready:
                    del p.grad_ready_hook
