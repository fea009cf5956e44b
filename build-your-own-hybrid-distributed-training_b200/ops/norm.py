"""Fused residual-add + LayerNorm / RMSNorm.

``add_norm(residual, delta, weight, bias)`` returns ``(r, y)`` with
``r = residual + delta`` kept in fp32 (the residual stream) and
``y = norm(r) * weight (+ bias)`` in the compute dtype, in one pass over the
row (``csrc/norm.cu``).  The backward kernel adds the gradient arriving on the
residual stream to the normalisation gradient, writes it once in fp32 (for the
residual) and once in the compute dtype (for the branch that produced
``delta``), and reduces the weight/bias gradients with per-CTA partial sums.

Parameters marked ``sequence_parallel_partial_grad`` still receive only this
rank's partial gradient; the hybrid model all-reduces them (reference
``src/hybrid_training/parallel/tensor_parallel.py:813-854``).
"""

from __future__ import annotations

from typing import Any

import torch
import torch.nn.functional as F

from ._ext import extension
from .grads import adopt_exposed_gradient, deliver_grad, has_main_grad, main_grad_beta

__all__ = ["add_norm", "layer_norm", "rms_norm"]


def _reference(residual: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor, bias: torch.Tensor | None,
               eps: float, rms: bool, out_dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    r = residual if delta is None else residual + delta.to(residual.dtype)
    rf = r.float()
    if rms:
        y = rf * torch.rsqrt(rf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
    else:
        y = F.layer_norm(rf, (rf.shape[-1],), weight.float(), None if bias is None else bias.float(), eps)
    return r, y.to(out_dtype)


class _AddNormFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, residual: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor,
                bias: torch.Tensor | None, eps: float, rms: bool, out_dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
        d = residual.shape[-1]
        rows = residual.numel() // d
        res2 = residual.reshape(rows, d)
        delta2 = None if delta is None else delta.reshape(rows, d)
        r = torch.empty(rows, d, dtype=torch.float32, device=residual.device)
        y = torch.empty(rows, d, dtype=out_dtype, device=residual.device)
        mean = torch.empty(rows, dtype=torch.float32, device=residual.device)
        rstd = torch.empty(rows, dtype=torch.float32, device=residual.device)
        extension().norm_forward(res2.contiguous(), None if delta2 is None else delta2.contiguous(), weight, bias, r, y,
                                 mean, rstd, float(eps), bool(rms))
        ctx.save_for_backward(r, weight, bias if bias is not None else r.new_empty(0), mean, rstd)
        ctx.has_bias, ctx.rms, ctx.has_delta = bias is not None, rms, delta is not None
        ctx.delta_dtype = None if delta is None else delta.dtype
        ctx.shape = residual.shape
        ctx.weight_param, ctx.bias_param = weight, bias
        return r.view(residual.shape), y.view(residual.shape)

    @staticmethod
    def backward(ctx: Any, dr: torch.Tensor | None, dy: torch.Tensor | None) -> tuple[Any, ...]:
        r, weight, bias, mean, rstd = ctx.saved_tensors
        rows, d = r.shape
        dy2 = None if dy is None else dy.reshape(rows, d).contiguous()
        dr2 = None if dr is None else dr.reshape(rows, d).contiguous()
        dres = torch.empty(rows, d, dtype=torch.float32, device=r.device)
        ddelta = torch.empty(rows, d, dtype=ctx.delta_dtype, device=r.device) if ctx.has_delta else None
        ext = extension()
        blocks = ext.norm_backward_blocks(rows)
        part_w = torch.empty(blocks, d, dtype=torch.float32, device=r.device)
        part_b = torch.empty(blocks, d, dtype=torch.float32, device=r.device) if ctx.has_bias else None
        ext.norm_backward(dy2, dr2, r, weight, mean, rstd, dres, ddelta, part_w, part_b, bool(ctx.rms))
        dw = db = None
        w, bp = ctx.weight_param, ctx.bias_param
        if ctx.has_bias and ctx.needs_input_grad[2] and ctx.needs_input_grad[3] and has_main_grad(w) and has_main_grad(bp):
            # Both reductions in one launch, straight into the two main_grad slices.
            adopt_exposed_gradient(w, from_autograd=False)
            adopt_exposed_gradient(bp, from_autograd=False)
            ext.sum_rows_pair(part_w, w.main_grad, main_grad_beta(w), part_b, bp.main_grad, main_grad_beta(bp))
            deliver_grad(w, compute=_written)
            deliver_grad(bp, compute=_written)
            return (dres.view(ctx.shape), None if ddelta is None else ddelta.view(ctx.shape), None, None, None, None, None)
        if ctx.needs_input_grad[2]:
            dw = deliver_grad(ctx.weight_param, compute=lambda out, beta: ext.sum_rows(part_w, out, beta),
                              value=None if getattr(ctx.weight_param, "main_grad", None) is not None else part_w.sum(0).to(ctx.weight_param.dtype))
        if ctx.has_bias and ctx.needs_input_grad[3]:
            db = deliver_grad(ctx.bias_param, compute=lambda out, beta: ext.sum_rows(part_b, out, beta),
                              value=None if getattr(ctx.bias_param, "main_grad", None) is not None else part_b.sum(0).to(ctx.bias_param.dtype))
        return (dres.view(ctx.shape), None if ddelta is None else ddelta.view(ctx.shape), dw, db, None, None, None)


def _written(out: torch.Tensor, beta: float) -> None:
    """Delivery of a gradient that a combined launch has already written into ``main_grad``."""


def add_norm(residual: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor, bias: torch.Tensor | None = None,
             *, eps: float = 1e-5, rms: bool = False, out_dtype: torch.dtype | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """``(residual + delta, norm(residual + delta))``; see the module docstring."""
    out_dtype = out_dtype or residual.dtype
    if not residual.is_cuda:
        return _reference(residual, delta, weight, bias, eps, rms, out_dtype)
    if residual.dtype != torch.float32:
        residual = residual.float()
    return _AddNormFunction.apply(residual, delta, weight, bias, eps, rms, out_dtype)


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, eps: float = 1e-5,
               out_dtype: torch.dtype | None = None) -> torch.Tensor:
    return add_norm(x, None, weight, bias, eps=eps, rms=False, out_dtype=out_dtype)[1]


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    return add_norm(x, None, weight, None, eps=eps, rms=True, out_dtype=out_dtype)[1]
