"""Fused optimizer and gradient-norm kernels over flat fp32 buffers.

``adamw_flat`` updates an fp32 master buffer, its two moment buffers and the
bf16 compute copy in one pass (``csrc/optim.cu``): each element is read once
and written once per buffer.  Hyper-parameters that change between steps
(learning rate, step count, gradient scale from clipping or loss scaling) are
read from a small device tensor, so a captured CUDA graph replays correctly.
The update is PyTorch's AdamW (decoupled weight decay, bias-corrected
moments), i.e. what ``src/hybrid_training/optim/sharded_optimizer.py:84-126``
builds with ``torch.optim.AdamW``.

``grad_sumsq`` accumulates the weighted squared gradient norm and a
non-finite flag in one pass (the distributed gradient norm, the fp16
overflow vote and clipping need no separate sweeps).
"""

from __future__ import annotations

import torch

from ._ext import extension

__all__ = ["HYPER_SLOTS", "adamw_flat", "grad_sumsq", "reference_adamw"]

# Layout of the device-side hyper-parameter vector.
HYPER_SLOTS = {"lr": 0, "step": 1, "grad_scale": 2, "skip": 3}


def reference_adamw(param: torch.Tensor, grad: torch.Tensor, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor, *, lr: float,
                    beta1: float, beta2: float, eps: float, weight_decay: float, step: int, grad_scale: float = 1.0) -> None:
    """In-place fp32 AdamW step in plain PyTorch (the CPU path and oracle)."""
    g = grad.float() * grad_scale
    param.mul_(1 - lr * weight_decay)
    exp_avg.mul_(beta1).add_(g, alpha=1 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    bc1 = 1 - beta1**step
    bc2 = 1 - beta2**step
    denom = (exp_avg_sq / bc2).sqrt_().add_(eps)
    param.addcdiv_(exp_avg, denom, value=-lr / bc1)


def adamw_flat(param: torch.Tensor, grad: torch.Tensor, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor,
               compute_copy: torch.Tensor | None, hyper: torch.Tensor, *, beta1: float, beta2: float, eps: float,
               weight_decay: float, resident: bool = False) -> None:
    """One fused AdamW step over flat CUDA buffers; ``hyper`` = ``[lr, step, grad_scale, skip]`` (fp32, device).

    ``resident=True`` launches the small-footprint form (one 128-thread block per SM) that runs
    beside a persistent GEMM, for slices updated during the backward pass.
    """
    extension().adamw_flat(param, grad, exp_avg, exp_avg_sq, compute_copy, hyper, float(beta1), float(beta2), float(eps),
                           float(weight_decay), bool(resident))


def grad_sumsq(grad: torch.Tensor, weights: torch.Tensor | None, out: torch.Tensor, scale: float = 1.0) -> None:
    """``out[0] += scale * sum(weights * grad^2)``; ``out[1] = 1`` if any element is non-finite (fp32 device)."""
    extension().grad_sumsq(grad, weights, out, float(scale))
