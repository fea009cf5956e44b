"""AdamW over one flat fp32 parameter space, updated by a single fused kernel.

At construction the optimizer lays its parameters out in one contiguous fp32
buffer (re-homing each ``param.data`` as a view) so that the update is one
kernel launch over the whole model instead of one per tensor:

* if every parameter already has a ``main_grad`` view into one flat gradient
  buffer (DDP's buckets), the parameter buffer mirrors that buffer's offsets,
  so element ``i`` of the parameters pairs with element ``i`` of the
  gradients;
* otherwise the optimizer allocates the flat gradient buffer itself and
  installs ``main_grad`` views, which the native backward kernels write into.

Moments (``exp_avg``, ``exp_avg_sq``) are flat buffers too, exposed per
parameter in ``state[param]`` as views, so ``state_dict`` has the usual
``torch.optim`` structure and the checkpoint format is unchanged.  On CUDA the
kernel also writes the bf16 compute copy of each weight (``param.compute_copy``)
that the forward GEMMs read, and takes the learning rate, step, gradient scale
(clipping / loss scaling) and skip flag from a device-side vector so the whole
step can be captured in a CUDA graph.  The arithmetic is PyTorch's AdamW.

Parameters that received no gradient in a step are updated with a zero
gradient (their moments decay and weight decay applies), whereas
``torch.optim.AdamW`` skips them; the training models here give every
parameter a gradient every step.
"""

from __future__ import annotations

import math
from collections.abc import Iterable
from typing import Any

import torch

from .. import ops

__all__ = ["FusedAdamW"]

_ALIGN = 64


def _common_storage(views: list[torch.Tensor]) -> torch.Tensor | None:
    """A 1-D tensor spanning the storage shared by ``views`` (or ``None`` if they do not share one)."""
    if not views or any(v is None for v in views):
        return None
    storage = views[0].untyped_storage()
    if any(v.untyped_storage().data_ptr() != storage.data_ptr() for v in views):
        return None
    dtype = views[0].dtype
    n = storage.nbytes() // torch.empty(0, dtype=dtype).element_size()
    return torch.empty(0, dtype=dtype, device=views[0].device).set_(storage, 0, (n,), (1,))


class FusedAdamW(torch.optim.Optimizer):
    """``torch.optim.AdamW`` semantics over a flat parameter space (see the module docstring)."""

    def __init__(self, params: Iterable[torch.nn.Parameter], lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 1e-2, *, compute_dtype: torch.dtype | None = None) -> None:
        unique: list[torch.nn.Parameter] = []
        seen: set[int] = set()
        for p in params:
            if p.requires_grad and id(p) not in seen:
                seen.add(id(p))
                unique.append(p)
        super().__init__(unique, dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay))
        self._params = unique
        device = unique[0].device
        self._device = device
        grads = [getattr(p, "main_grad", None) for p in unique]
        shared = _common_storage(grads)  # type: ignore[arg-type]
        if shared is not None and shared.dtype == torch.float32:
            self._grad_flat = shared
            offsets = [g.storage_offset() for g in grads]  # type: ignore[union-attr]
        else:
            offsets, total = [], 0
            for p in unique:
                offsets.append(total)
                total += -(-p.numel() // _ALIGN) * _ALIGN
            self._grad_flat = torch.zeros(total, dtype=torch.float32, device=device)
            for p, off in zip(unique, offsets):
                p.main_grad = self._grad_flat[off:off + p.numel()].view(p.shape)
                p.main_grad_fresh = True
        self._offsets = offsets
        n = self._grad_flat.numel()
        self._param_flat = torch.zeros(n, dtype=torch.float32, device=device)
        with torch.no_grad():
            for p, off in zip(unique, offsets):
                self._param_flat[off:off + p.numel()].copy_(p.detach().reshape(-1))
                p.data = self._param_flat[off:off + p.numel()].view(p.shape)
        self._exp_avg = torch.zeros_like(self._param_flat)
        self._exp_avg_sq = torch.zeros_like(self._param_flat)
        self._step_count = 0
        for p, off in zip(unique, offsets):
            self.state[p] = {
                "step": torch.tensor(0.0),
                "exp_avg": self._exp_avg[off:off + p.numel()].view(p.shape),
                "exp_avg_sq": self._exp_avg_sq[off:off + p.numel()].view(p.shape),
            }
        self._compute_flat: torch.Tensor | None = None
        if compute_dtype is not None and compute_dtype != torch.float32 and device.type == "cuda":
            self._compute_flat = self._param_flat.to(compute_dtype)
            for p, off in zip(unique, offsets):
                p.compute_copy = self._compute_flat[off:off + p.numel()].view(p.shape)
                p.compute_copy_version = p._version
        # [lr, step, grad_scale, skip]; refreshed from the host (pinned) every step.
        self._hyper_host = torch.zeros(4, dtype=torch.float32, pin_memory=device.type == "cuda")
        self._hyper = torch.zeros(4, dtype=torch.float32, device=device)
        self._grad_scale_device: torch.Tensor | None = None
        # Recorded after each eager host-to-device copy of the staging buffer: the host must not
        # overwrite the pinned buffer while that copy may still be queued.
        self._hyper_copied: torch.cuda.Event | None = None

    # -- flat views ---------------------------------------------------------------------------------
    @property
    def flat_parameters(self) -> torch.Tensor:
        return self._param_flat

    @property
    def flat_gradients(self) -> torch.Tensor:
        return self._grad_flat

    @property
    def hyper_parameters(self) -> torch.Tensor:
        """Device vector ``[lr, step, grad_scale, skip]`` read by the kernel."""
        return self._hyper

    def set_device_grad_scale(self, scale: torch.Tensor | None) -> None:
        """Use a device scalar (e.g. the clip coefficient) as the gradient multiplier of the next steps."""
        self._grad_scale_device = scale

    def refresh_compute_copies(self) -> None:
        """Re-cast the compute copies after the fp32 parameters were changed outside :meth:`step`."""
        if self._compute_flat is not None:
            with torch.no_grad():
                self._compute_flat.copy_(self._param_flat)
            for p in self._params:
                p.compute_copy_version = p._version

    def _collect_autograd_grads(self) -> None:
        """Move gradients that arrived through plain autograd into the flat buffer."""
        for p in self._params:
            g = p.grad
            mg = p.main_grad
            if g is not None and g.data_ptr() != mg.data_ptr():
                mg.copy_(g.detach().reshape(mg.shape))
                p.main_grad_fresh = False
            elif g is None and getattr(p, "main_grad_fresh", False):
                mg.zero_()

    def prepare_step(self) -> None:
        """Host half of a step: advance the step count and stage ``[lr, step, 1, 0]`` in pinned memory.

        A captured CUDA graph replays :meth:`launch_step`, which reads this staging
        buffer, so calling ``prepare_step`` before each replay is what advances the
        schedule inside the graph.
        """
        group = self.param_groups[0]
        self._step_count += 1
        for p in self._params:
            self.state[p]["step"].fill_(float(self._step_count))
        if self._hyper_copied is not None:
            self._hyper_copied.synchronize()
        self._hyper_host.copy_(torch.tensor([group["lr"], float(self._step_count), 1.0, 0.0]))

    @torch.no_grad()
    def stage_hyper_parameters(self) -> None:
        """Copy the staged ``[lr, step, grad_scale, skip]`` to the device vector (stream-ordered, no host sync).

        :meth:`launch_step` does this itself; kernels that apply the update elsewhere (the FSDP
        reduce-scatter + AdamW kernel) call it before they run.
        """
        self._hyper.copy_(self._hyper_host, non_blocking=True)
        if self._hyper.is_cuda and not torch.cuda.is_current_stream_capturing():
            if self._hyper_copied is None:
                self._hyper_copied = torch.cuda.Event()
            self._hyper_copied.record()
        if self._grad_scale_device is not None:
            self._hyper[2:3].copy_(self._grad_scale_device.reshape(1))

    @torch.no_grad()
    def launch_step(self, deferred: tuple[int, int, Any] | None = None) -> None:
        """Device half of a step (CUDA): one fused kernel over the flat buffers; no host synchronisation.

        ``deferred = (start, numel, wait)``: the gradients in ``[start, start + numel)`` of the flat
        buffer are still being reduced; every other element is updated first, then ``wait()`` makes
        the stream wait for that reduction and the range is updated last, so the update of the rest
        overlaps the last reduction.
        """
        group = self.param_groups[0]
        beta1, beta2 = group["betas"]
        self._collect_autograd_grads()
        self.stage_hyper_parameters()

        def update(lo: int, hi: int) -> None:
            if hi <= lo:
                return
            copy = None if self._compute_flat is None else self._compute_flat[lo:hi]
            ops.adamw_flat(self._param_flat[lo:hi], self._grad_flat[lo:hi], self._exp_avg[lo:hi], self._exp_avg_sq[lo:hi], copy,
                           self._hyper, beta1=beta1, beta2=beta2, eps=group["eps"], weight_decay=group["weight_decay"])

        if deferred is None:
            update(0, self._param_flat.numel())
        else:
            start, numel, wait = deferred
            total = self._param_flat.numel()
            end = min(total, start + -(-numel // _ALIGN) * _ALIGN)
            update(0, start)
            update(end, total)
            wait()
            update(start, end)
        if self._compute_flat is not None:
            for p in self._params:
                p.compute_copy_version = p._version

    @torch.no_grad()
    def step(self, closure: Any = None) -> Any:
        loss = closure() if closure is not None else None
        self.prepare_step()
        if self._param_flat.is_cuda:
            self.launch_step()
            return loss
        group = self.param_groups[0]
        beta1, beta2 = group["betas"]
        self._collect_autograd_grads()
        scale = 1.0 if self._grad_scale_device is None else float(self._grad_scale_device)
        _adamw_reference_flat(self._param_flat, self._grad_flat, self._exp_avg, self._exp_avg_sq, lr=group["lr"],
                              beta1=beta1, beta2=beta2, eps=group["eps"], weight_decay=group["weight_decay"],
                              step=self._step_count, grad_scale=scale)
        return loss

    def zero_grad(self, set_to_none: bool = True) -> None:
        for p in self._params:
            p.grad = None
            p.main_grad_fresh = True

    # -- state dict: keep the flat views alive --------------------------------------------------------
    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        groups = state_dict["param_groups"]
        for mine, saved in zip(self.param_groups, groups):
            for k, v in saved.items():
                if k != "params":
                    mine[k] = tuple(v) if k == "betas" else v
        saved_state = state_dict["state"]
        step = 0
        with torch.no_grad():
            for index, p in enumerate(self._params):
                entry = saved_state.get(index, saved_state.get(str(index)))
                if not entry:
                    continue
                for key in ("exp_avg", "exp_avg_sq"):
                    if key in entry:
                        self.state[p][key].copy_(torch.as_tensor(entry[key]).reshape(p.shape).to(self.state[p][key]))
                if "step" in entry:
                    step = int(float(torch.as_tensor(entry["step"]).item()))
                    self.state[p]["step"].fill_(float(step))
        self._step_count = step
        self.refresh_compute_copies()


def _adamw_reference_flat(param: torch.Tensor, grad: torch.Tensor, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor, *, lr: float,
                          beta1: float, beta2: float, eps: float, weight_decay: float, step: int, grad_scale: float) -> None:
    """PyTorch's single-tensor AdamW arithmetic on the flat buffers (CPU path)."""
    g = grad if grad_scale == 1.0 else grad * grad_scale
    param.mul_(1 - lr * weight_decay)
    exp_avg.lerp_(g, 1 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    bc1 = 1 - beta1**step
    bc2 = 1 - beta2**step
    denom = (exp_avg_sq.sqrt() / math.sqrt(bc2)).add_(eps)
    param.addcdiv_(exp_avg, denom, value=-lr / bc1)
