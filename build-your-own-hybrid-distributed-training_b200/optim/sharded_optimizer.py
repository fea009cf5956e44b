"""Optimizer over the local (possibly sharded) parameters, with a distributed gradient norm.

API and semantics of ``src/hybrid_training/optim/sharded_optimizer.py:84-499``:
the inner optimizer sees only this rank's parameters (flat shards under FSDP,
so its state is sharded too); the global gradient norm weights every local
element by ``multiplicity / world`` -- a replicated element is counted once
across the world, a tensor-parallel or FSDP shard once per owner -- and is
all-reduced over the world group; ``clip_grad_norm`` rescales gradients when
the norm exceeds the limit; optional CPU offload keeps master copies and
optimizer state on the host.

Differences: AdamW is :class:`FusedAdamW` (one kernel over a flat parameter
space); the weighted sum of squares runs as one pass over the flat gradient
buffer; and clipping never synchronises with the host: the coefficient stays
on the device and is applied inside the AdamW kernel (the gradients are not
rescaled in place on CUDA).
"""

from __future__ import annotations

from collections.abc import Iterable, Sequence
from dataclasses import dataclass
from typing import Any

import torch
import torch.nn as nn

from .. import ops
from ..config import OptimizerConfig
from ..distributed.collectives import CommunicationRecorder, ReduceOp, all_reduce
from ..distributed.groups import GroupHandle
from ..errors import ShardingError, format_error
from ..logging import get_logger
from .fused_adamw import FusedAdamW

__all__ = ["NormContribution", "ShardedOptimizer", "build_gradient_norm_contributions", "build_inner_optimizer",
           "distributed_gradient_norm"]

_LOG = get_logger(__name__)


def build_inner_optimizer(parameters: Iterable[nn.Parameter], config: OptimizerConfig, *,
                          compute_dtype: torch.dtype | None = None, fused: bool = True) -> torch.optim.Optimizer:
    """AdamW (flat, fused) or SGD over the trainable parameters."""
    params = [p for p in parameters if p.requires_grad]
    if not params:
        raise ShardingError(format_error("optim.build_inner_optimizer", "the optimizer was given nothing to train",
                                         expected="one or more parameters that require gradients", observed=0,
                                         resolution="wrap the model before building the optimizer"))
    b1, b2 = float(config.betas[0]), float(config.betas[1])
    if config.name == "adamw":
        if fused:
            return FusedAdamW(params, lr=config.learning_rate, betas=(b1, b2), eps=config.eps,
                              weight_decay=config.weight_decay, compute_dtype=compute_dtype)
        return torch.optim.AdamW(params, lr=config.learning_rate, betas=(b1, b2), eps=config.eps, weight_decay=config.weight_decay)
    return torch.optim.SGD(params, lr=config.learning_rate, momentum=config.momentum, weight_decay=config.weight_decay)


@dataclass
class NormContribution:
    """One parameter's weighted contribution to the squared global norm."""

    parameter: nn.Parameter
    scale: float | torch.Tensor
    label: str

    def squared_norm(self) -> torch.Tensor:
        grad = _grad_of(self.parameter)
        if grad is None:
            return torch.zeros((), dtype=torch.float64)
        sq = grad.detach().double().pow(2)
        if isinstance(self.scale, torch.Tensor):
            return (sq.reshape(-1) * self.scale.to(device=sq.device, dtype=torch.float64)).sum()
        return sq.sum() * float(self.scale)


def _grad_of(p: nn.Parameter) -> torch.Tensor | None:
    if p.grad is not None:
        return p.grad
    mg = getattr(p, "main_grad", None)
    return None if mg is None or getattr(p, "main_grad_fresh", True) else mg


def build_gradient_norm_contributions(parameters: Sequence[nn.Parameter], *, world_size: int) -> list[NormContribution]:
    if world_size < 1:
        raise ShardingError(format_error("optim.build_gradient_norm_contributions", "the reduction group has at least one rank", expected=">= 1",
                                         observed=world_size, resolution="give the number of ranks in the norm group"))
    out = []
    for i, p in enumerate(parameters):
        vector = getattr(p, "gradient_norm_scale_vector", None)
        if vector is not None:
            out.append(NormContribution(p, vector.double() / world_size, getattr(p, "gradient_norm_label", f"flat_param#{i}")))
            continue
        multiplicity = 1 if getattr(p, "is_tensor_parallel_replicated", True) else int(getattr(p, "tensor_parallel_group_size", 1))
        out.append(NormContribution(p, multiplicity / world_size, f"param#{i}"))
    return out


def distributed_gradient_norm(contributions: Sequence[NormContribution], group: GroupHandle, *, device: torch.device,
                              recorder: CommunicationRecorder | None = None) -> torch.Tensor:
    """``sqrt(sum over ranks of weighted local squared norms)`` as a device fp64 scalar."""
    total = torch.zeros((), dtype=torch.float64, device=device)
    for c in contributions:
        total = total + c.squared_norm().to(device)
    buf = total.reshape(1).contiguous()
    all_reduce(buf, group, op=ReduceOp.SUM, recorder=recorder).wait()
    return buf[0].clamp_min(0).sqrt()


class ShardedOptimizer:
    """The inner optimizer plus distributed clipping, LR control, offload and state (see module docstring)."""

    def __init__(self, parameters: Iterable[nn.Parameter], config: OptimizerConfig, *, norm_group: GroupHandle,
                 device: torch.device, recorder: CommunicationRecorder | None = None,
                 compute_dtype: torch.dtype | None = None) -> None:
        self._parameters = [p for p in parameters if p.requires_grad]
        self._config, self._norm_group, self._device, self._recorder = config, norm_group, device, recorder
        self._offload = config.cpu_offload_state and device.type != "cpu"
        if self._offload:
            self._cpu_parameters = [nn.Parameter(p.detach().cpu().clone(), requires_grad=True) for p in self._parameters]
            self._optimizer = build_inner_optimizer(self._cpu_parameters, config, fused=False)
        else:
            self._cpu_parameters = []
            self._optimizer = build_inner_optimizer(self._parameters, config, compute_dtype=compute_dtype)
        self._contributions = build_gradient_norm_contributions(self._parameters, world_size=norm_group.size)
        self._norm_weights: torch.Tensor | None = None
        self._norm_buffer: torch.Tensor | None = None

    # -- gradient norm ------------------------------------------------------------------------------------
    def _flat_norm_weights(self) -> torch.Tensor:
        """Per-element weight vector aligned with the fused optimizer's flat gradient buffer."""
        if self._norm_weights is None:
            inner = self._optimizer
            assert isinstance(inner, FusedAdamW)
            w = torch.zeros(inner.flat_gradients.numel(), dtype=torch.float32, device=self._device)
            for c, p in zip(self._contributions, self._parameters):
                off = p.main_grad.storage_offset()
                n = p.numel()
                if isinstance(c.scale, torch.Tensor):
                    w[off:off + n] = c.scale.to(device=self._device, dtype=torch.float32)
                else:
                    w[off:off + n] = float(c.scale)
            self._norm_weights = w
        return self._norm_weights

    def gradient_norm(self) -> torch.Tensor:
        """The global gradient norm as a device scalar (fp64 on CPU, fp32 on CUDA); no host synchronisation."""
        inner = self._optimizer
        if isinstance(inner, FusedAdamW) and inner.flat_gradients.is_cuda:
            inner._collect_autograd_grads()
            if self._norm_buffer is None:
                self._norm_buffer = torch.zeros(2, dtype=torch.float32, device=self._device)
            self._norm_buffer.zero_()
            ops.grad_sumsq(inner.flat_gradients, self._flat_norm_weights(), self._norm_buffer)
            all_reduce(self._norm_buffer, self._norm_group, op=ReduceOp.SUM, recorder=self._recorder).wait()
            return self._norm_buffer[0].clamp_min(0).sqrt()
        return distributed_gradient_norm(self._contributions, self._norm_group, device=self._device, recorder=self._recorder)

    def clip_grad_norm(self, max_norm: float) -> torch.Tensor:
        """Compute the global norm and, if ``max_norm > 0``, scale gradients by ``min(1, max_norm / (norm + 1e-6))``."""
        norm = self.gradient_norm()
        if max_norm <= 0:
            return norm
        coefficient = (max_norm / (norm.float() + 1e-6)).clamp(max=1.0)
        inner = self._optimizer
        if isinstance(inner, FusedAdamW) and inner.flat_gradients.is_cuda:
            inner.set_device_grad_scale(coefficient)
        else:
            c = float(coefficient)
            if c < 1.0:
                for p in self._parameters:
                    g = _grad_of(p)
                    if g is not None:
                        g.detach().mul_(c)
        return norm

    # -- stepping ---------------------------------------------------------------------------------------
    def step(self) -> None:
        if self._offload:
            for dp, cp in zip(self._parameters, self._cpu_parameters):
                g = _grad_of(dp)
                if g is None:
                    cp.grad = None
                else:
                    if cp.grad is None:
                        cp.grad = torch.empty_like(cp)
                    cp.grad.copy_(g.detach().cpu())
            self._optimizer.step()
            with torch.no_grad():
                for dp, cp in zip(self._parameters, self._cpu_parameters):
                    dp.data.copy_(cp.data.to(dp.device))
            return
        self._optimizer.step()

    def zero_grad(self, *, set_to_none: bool = True) -> None:
        for p in self._parameters:
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.detach().zero_()
            if getattr(p, "main_grad", None) is not None:
                p.main_grad_fresh = True
        if isinstance(self._optimizer, FusedAdamW):
            self._optimizer.set_device_grad_scale(None)
        for p in self._cpu_parameters:
            p.grad = None

    # -- accessors / state --------------------------------------------------------------------------------
    parameters = property(lambda self: tuple(self._parameters))
    inner = property(lambda self: self._optimizer)
    norm_group = property(lambda self: self._norm_group)

    @property
    def learning_rate(self) -> float:
        return float(self._optimizer.param_groups[0]["lr"])

    def set_learning_rate(self, value: float) -> None:
        for g in self._optimizer.param_groups:
            g["lr"] = value

    def state_bytes(self) -> int:
        if isinstance(self._optimizer, FusedAdamW):
            return 2 * self._optimizer.flat_parameters.numel() * 4
        return sum(v.numel() * v.element_size() for s in self._optimizer.state.values() for v in s.values() if torch.is_tensor(v))

    def state_dict(self) -> dict[str, Any]:
        inner = self._optimizer.state_dict()
        state = {int(i): {k: v.detach().cpu().clone() if torch.is_tensor(v) else v for k, v in e.items()}
                 for i, e in inner["state"].items()}
        return {"param_groups": [{k: v for k, v in g.items() if k != "params"} for g in inner["param_groups"]],
                "state": state, "num_parameters": len(self._parameters)}

    def load_state_dict(self, payload: dict[str, Any]) -> None:
        expected, observed = len(self._parameters), int(payload.get("num_parameters", -1))
        if observed != expected:
            raise ShardingError(format_error("optim.load_state_dict", "the saved optimizer state does not match this "
                                             "optimizer's parameter count", rank=self._norm_group.global_rank, expected=expected, observed=observed,
                                             resolution="restore into the same model, wrapped into the same units"))
        target = self._cpu_parameters if self._offload else self._parameters
        groups = []
        for saved, existing in zip(payload["param_groups"], self._optimizer.state_dict()["param_groups"]):
            merged = dict(existing)
            merged.update(saved)
            merged["params"] = existing["params"]
            groups.append(merged)
        state = {}
        for i, entry in payload["state"].items():
            ref = target[int(i)]
            state[int(i)] = {k: v.to(device=ref.device, dtype=ref.dtype) if torch.is_tensor(v) and v.is_floating_point() and v.numel() > 1
                             else v for k, v in entry.items()}
        self._optimizer.load_state_dict({"state": state, "param_groups": groups})

    def refresh_compute_copies(self) -> None:
        if isinstance(self._optimizer, FusedAdamW):
            self._optimizer.refresh_compute_copies()

    @property
    def offloaded(self) -> bool:
        """Whether the master parameters and optimizer state live in host memory."""
        return self._offload

    def __repr__(self) -> str:
        return (f"ShardedOptimizer({self._config.name}, params={len(self._parameters)}, norm_group={self._norm_group.name!r}, "
                f"offload={self._offload})")
