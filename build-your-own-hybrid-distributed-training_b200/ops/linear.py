"""GEMM and the fused linear layer.

``gemm`` is the entry point to the tcgen05 GEMM (``csrc/gemm_tcgen05.cu``):
``D = epilogue(op(A) @ op(B)^T + bias) (+ beta * D)`` with bf16 operands, fp32
accumulation in tensor memory and one of these epilogues:

* ``PLAIN``    -- store ``acc (+ bias)``;
* ``GELU``     -- store ``gelu_tanh(acc + bias)`` and, into ``aux``, the pre-activation;
* ``GELU_BWD`` -- store ``acc * gelu_tanh'(aux)`` (activation backward fused into dgrad);
* ``beta=1``   -- accumulate into an fp32 ``D`` (gradient accumulation into ``main_grad``).

Operand majorness follows the three GEMMs of a linear layer ``Y = X W^T``:
forward (A=X, B=W, both K-major), dgrad ``dX = dY W`` (B is W read MN-major)
and wgrad ``dW = dY^T X`` (both read MN-major), so no operand is ever
transposed in memory.

On CPU tensors the same functions run in fp32 PyTorch; that path is also the
numerical oracle for the kernel tests.
"""

from __future__ import annotations

import math
from typing import Any

import torch
import torch.nn.functional as F

from ._ext import extension
from .grads import deliver_grad

__all__ = ["EPI_GELU", "EPI_GELU_BWD", "EPI_PLAIN", "compute_weight", "gelu_backward", "gelu_mlp", "gemm", "linear",
           "reference_gemm", "swiglu", "swiglu_gemm", "swiglu_mlp", "swiglu_mlp_supported"]

EPI_PLAIN = 0
EPI_GELU = 1
EPI_GELU_BWD = 2

_SQRT_2_OVER_PI = math.sqrt(2.0 / math.pi)


def _gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return F.gelu(x, approximate="tanh")


def _gelu_tanh_grad(x: torch.Tensor) -> torch.Tensor:
    x = x.float()
    inner = _SQRT_2_OVER_PI * (x + 0.044715 * x**3)
    t = torch.tanh(inner)
    return 0.5 * (1 + t) + 0.5 * x * (1 - t * t) * _SQRT_2_OVER_PI * (1 + 3 * 0.044715 * x * x)


def reference_gemm(a: torch.Tensor, b: torch.Tensor, *, a_mn_major: bool = False, b_mn_major: bool = False,
                   bias: torch.Tensor | None = None, aux: torch.Tensor | None = None, epilogue: int = EPI_PLAIN,
                   c: torch.Tensor | None = None, beta: float = 0.0,
                   alpha: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor | None]:
    """fp32 PyTorch statement of :func:`gemm` (returns ``(d, aux_out)``)."""
    A = (a.t() if a_mn_major else a).float()
    B = (b.t() if b_mn_major else b).float()
    acc = A @ B.t()
    if alpha is not None:
        acc = acc * alpha.float().reshape(())
    if bias is not None:
        acc = acc + bias.float()
    aux_out = None
    if epilogue == EPI_GELU:
        aux_out = acc
        acc = _gelu_tanh(acc)
    elif epilogue == EPI_GELU_BWD:
        acc = acc * _gelu_tanh_grad(aux)
    if c is not None and beta != 0.0:
        acc = acc + beta * c.float()
    return acc, aux_out


def gemm(a: torch.Tensor, b: torch.Tensor, *, out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
         a_mn_major: bool = False, b_mn_major: bool = False, bias: torch.Tensor | None = None,
         aux: torch.Tensor | None = None, epilogue: int = EPI_PLAIN, beta: float = 0.0,
         alpha: torch.Tensor | None = None) -> torch.Tensor:
    """``D[M,N] = epi(alpha * op(A) op(B)^T + bias) + beta*D``.

    ``alpha`` is an optional one-element fp32 device tensor (read by the kernel,
    so the scale never crosses to the host).

    ``a`` is ``[M,K]`` (K-major) or ``[K,M]`` (``a_mn_major``); ``b`` is ``[N,K]``
    or ``[K,N]`` (``b_mn_major``).  ``out`` may be a row-padded view.
    """
    m = a.shape[1] if a_mn_major else a.shape[0]
    n = b.shape[1] if b_mn_major else b.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=out_dtype or a.dtype, device=a.device)
    if not a.is_cuda:
        d, aux_out = reference_gemm(a, b, a_mn_major=a_mn_major, b_mn_major=b_mn_major, bias=bias, aux=aux,
                                    epilogue=epilogue, c=out if beta else None, beta=beta, alpha=alpha)
        out.copy_(d)
        if aux_out is not None and aux is not None:
            aux.copy_(aux_out)
        return out
    extension().gemm(a, b, out, bias, aux, alpha, bool(a_mn_major), bool(b_mn_major), int(epilogue), float(beta))
    return out


def set_deterministic_reductions(on: bool) -> None:
    """Choose fixed-order split-K sums (bitwise reproducible, the default) or direct fp32 reduce-adds (faster).

    Affects the native GEMM's split-K path for fp32 outputs (weight gradients): with ``on=False`` every
    partial tile is added into the output by TMA reduce-adds, so no workspace or reduction pass is
    needed, but the order of the additions, and so the last bits, varies between runs.
    """
    extension().set_deterministic_reductions(bool(on))


def gelu_backward(grad: torch.Tensor, pre: torch.Tensor) -> torch.Tensor:
    """``grad * gelu_tanh'(pre)`` (bf16 in, bf16 out on CUDA)."""
    if not grad.is_cuda:
        return (grad.float() * _gelu_tanh_grad(pre)).to(grad.dtype)
    out = torch.empty_like(grad)
    extension().gelu_backward(grad.contiguous(), pre.contiguous(), out)
    return out


def compute_weight(weight: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """The ``dtype`` copy of an fp32 master weight.

    The fused optimizer keeps ``weight.compute_copy`` up to date in the same
    kernel that updates the master; any other in-place change (checkpoint load,
    broadcast) bumps the version counter and the copy is re-made here.
    """
    if weight.dtype == dtype:
        return weight
    copy = getattr(weight, "compute_copy", None)
    if copy is not None and copy.dtype == dtype and getattr(weight, "compute_copy_version", -1) == weight._version:
        return copy
    if copy is not None and copy.dtype == dtype:
        with torch.no_grad():
            copy.copy_(weight)
        weight.compute_copy_version = weight._version
        return copy
    return weight.detach().to(dtype)


def _column_sum(x: torch.Tensor, out: torch.Tensor | None = None, beta: float = 0.0) -> torch.Tensor:
    """fp32 sum over rows (the bias gradient), written as ``out = sum + beta * out``."""
    if not x.is_cuda:
        s = x.float().sum(0)
        if out is None:
            return s
        out.mul_(beta).add_(s) if beta else out.copy_(s)
        return out
    if out is None:
        out = torch.empty(x.shape[1], dtype=torch.float32, device=x.device)
    extension().column_sum(x, out, float(beta))
    return out


class _LinearFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, gelu: bool) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        w = compute_weight(weight, x.dtype)
        n = w.shape[0]
        y = torch.empty(x2.shape[0], n, dtype=x.dtype, device=x.device)
        pre = None
        if gelu:
            pre = torch.empty_like(y)
            gemm(x2, w, out=y, bias=bias, aux=pre, epilogue=EPI_GELU)
        else:
            gemm(x2, w, out=y, bias=bias)
        ctx.save_for_backward(x2, w, pre)
        ctx.weight, ctx.bias, ctx.gelu = weight, bias, gelu
        return y.view(*lead, n)

    @staticmethod
    def backward(ctx: Any, dy: torch.Tensor) -> tuple[Any, ...]:
        x2, w, pre = ctx.saved_tensors
        weight, bias = ctx.weight, ctx.bias
        dy2 = dy.reshape(-1, dy.shape[-1])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        g = gelu_backward(dy2, pre) if ctx.gelu else dy2
        dx = None
        if ctx.needs_input_grad[0]:
            dx = gemm(g, w, b_mn_major=True).view(*dy.shape[:-1], w.shape[1])
        dw = db = None
        if ctx.needs_input_grad[1]:
            dw = deliver_grad(weight, compute=lambda out, beta: gemm(g, x2, out=out, a_mn_major=True, b_mn_major=True,
                                                                      beta=beta),
                              value=None if getattr(weight, "main_grad", None) is not None else
                              gemm(g, x2, out_dtype=weight.dtype, a_mn_major=True, b_mn_major=True))
        if bias is not None and ctx.needs_input_grad[2]:
            db = deliver_grad(bias, compute=lambda out, beta: _column_sum(g, out, beta),
                              value=None if getattr(bias, "main_grad", None) is not None else _column_sum(g).to(bias.dtype))
        return dx, dw, db, None


class _GeluMLPFunction(torch.autograd.Function):
    """``fc2(gelu(fc1(x)))`` with the GELU derivative applied inside fc2's data-gradient GEMM.

    Forward: the fc1 GEMM epilogue adds the bias, stores the pre-activation and applies the GELU;
    backward: the fc2 data-gradient GEMM multiplies by gelu'(pre) in its epilogue, so the
    gradient at fc1's output is produced directly (no separate element-wise pass over the
    hidden activations).
    """

    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor | None, w2: torch.Tensor,
                b2: torch.Tensor | None) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        w1c, w2c = compute_weight(w1, x.dtype), compute_weight(w2, x.dtype)
        h = torch.empty(x2.shape[0], w1c.shape[0], dtype=x.dtype, device=x.device)
        pre = torch.empty_like(h)
        gemm(x2, w1c, out=h, bias=b1, aux=pre, epilogue=EPI_GELU)
        y = gemm(h, w2c, bias=b2)
        ctx.save_for_backward(x2, w1c, w2c, h, pre)
        ctx.params = (w1, b1, w2, b2)
        return y.view(*lead, w2c.shape[0])

    @staticmethod
    def backward(ctx: Any, dy: torch.Tensor) -> tuple[Any, ...]:
        x2, w1c, w2c, h, pre = ctx.saved_tensors
        w1, b1, w2, b2 = ctx.params
        dy2 = dy.reshape(-1, dy.shape[-1])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        g = gemm(dy2, w2c, b_mn_major=True, aux=pre, epilogue=EPI_GELU_BWD)

        def weight_grad(param: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor | None:
            return deliver_grad(param, compute=lambda out, beta: gemm(a, b, out=out, a_mn_major=True, b_mn_major=True, beta=beta),
                                value=None if getattr(param, "main_grad", None) is not None else
                                gemm(a, b, out_dtype=param.dtype, a_mn_major=True, b_mn_major=True))

        def bias_grad(param: torch.Tensor | None, a: torch.Tensor) -> torch.Tensor | None:
            if param is None:
                return None
            return deliver_grad(param, compute=lambda out, beta: _column_sum(a, out, beta),
                                value=None if getattr(param, "main_grad", None) is not None else _column_sum(a).to(param.dtype))

        dw2 = weight_grad(w2, dy2, h) if ctx.needs_input_grad[3] else None
        db2 = bias_grad(b2, dy2) if ctx.needs_input_grad[4] else None
        dx = gemm(g, w1c, b_mn_major=True).view(*dy.shape[:-1], w1c.shape[1]) if ctx.needs_input_grad[0] else None
        dw1 = weight_grad(w1, g, x2) if ctx.needs_input_grad[1] else None
        db1 = bias_grad(b1, g) if ctx.needs_input_grad[2] else None
        return dx, dw1, db1, dw2, db2


def gelu_mlp(x: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor | None, w2: torch.Tensor, b2: torch.Tensor | None) -> torch.Tensor:
    """``gelu(x w1^T + b1) w2^T + b2`` (tanh GELU) with both GELU passes fused into GEMM epilogues on CUDA."""
    if not x.is_cuda:
        h = _gelu_tanh(F.linear(x, w1.to(x.dtype), None if b1 is None else b1.to(x.dtype)))
        return F.linear(h, w2.to(x.dtype), None if b2 is None else b2.to(x.dtype))
    return _GeluMLPFunction.apply(x, w1, b1, w2, b2)


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *, activation: str | None = None) -> torch.Tensor:
    """``activation(x @ weight^T + bias)`` in the compute dtype of ``x`` with fp32 master weights.

    ``activation`` is ``None`` or ``'gelu'`` (tanh approximation) -- the GELU is
    fused into the GEMM epilogue on CUDA.
    """
    if activation not in (None, "gelu"):
        raise ValueError(f"linear supports activation None or 'gelu', got {activation!r}")
    if not x.is_cuda:
        y = F.linear(x, weight.to(x.dtype), None if bias is None else bias.to(x.dtype))
        return _gelu_tanh(y) if activation == "gelu" else y
    return _LinearFunction.apply(x, weight, bias, activation == "gelu")


class _SwiGLUFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, h: torch.Tensor) -> torch.Tensor:
        h = h.contiguous()
        f = h.shape[-1] // 2
        out = torch.empty(*h.shape[:-1], f, dtype=h.dtype, device=h.device)
        extension().swiglu_forward(h, out)
        ctx.save_for_backward(h)
        return out

    @staticmethod
    def backward(ctx: Any, grad: torch.Tensor) -> torch.Tensor:
        (h,) = ctx.saved_tensors
        dh = torch.empty_like(h)
        extension().swiglu_backward(h, grad.contiguous(), dh)
        return dh


def swiglu_gemm(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """``(h, a)``: ``h = x w^T + bias`` as ``[gate | up]`` and ``a = silu(gate) * up``, from one GEMM on CUDA.

    ``w`` is ``[2F, K]`` (gate rows, then up rows) in the compute dtype; ``F`` a multiple of 128.
    """
    m, f = x.shape[0], w.shape[0] // 2
    h = torch.empty(m, 2 * f, dtype=x.dtype, device=x.device)
    a = torch.empty(m, f, dtype=x.dtype, device=x.device)
    extension().gemm_swiglu(x, w, h, a, bias, False)
    return h, a


def _swiglu_dgrad(dy: torch.Tensor, w2: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
    """``dH = [dA * up * silu'(gate) | dA * silu(gate)]`` with ``dA = dy w2``, from one GEMM."""
    dh = torch.empty_like(h)
    extension().gemm_swiglu(dy, w2, h, dh, None, True)
    return dh


class _SwiGLUMLPFunction(torch.autograd.Function):
    """``fc2(silu(gate) * up)`` with ``[gate | up] = fc1(x)``, the activation inside two GEMM epilogues.

    Forward: fc1's GEMM loads the gate rows and the up rows of the weight into one 256-wide tile,
    stores the pre-activations (needed by the backward pass) and the activation in its epilogue;
    backward: fc2's data-gradient GEMM reads the pre-activations back and writes the gradient at
    fc1's output directly.  Compared with an element-wise SwiGLU kernel on each side this removes
    one write and one read of ``[M, 2F]`` plus one read and one write of ``[M, F]`` per pass.
    """

    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor | None, w2: torch.Tensor,
                b2: torch.Tensor | None) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        w1c, w2c = compute_weight(w1, x.dtype), compute_weight(w2, x.dtype)
        h, a = swiglu_gemm(x2, w1c, b1)
        y = gemm(a, w2c, bias=b2)
        ctx.save_for_backward(x2, w1c, w2c, h, a)
        ctx.params = (w1, b1, w2, b2)
        return y.view(*lead, w2c.shape[0])

    @staticmethod
    def backward(ctx: Any, dy: torch.Tensor) -> tuple[Any, ...]:
        x2, w1c, w2c, h, a = ctx.saved_tensors
        w1, b1, w2, b2 = ctx.params
        dy2 = dy.reshape(-1, dy.shape[-1])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dh = _swiglu_dgrad(dy2, w2c, h)

        def weight_grad(param: torch.Tensor, lhs: torch.Tensor, rhs: torch.Tensor) -> torch.Tensor | None:
            return deliver_grad(param, compute=lambda out, beta: gemm(lhs, rhs, out=out, a_mn_major=True, b_mn_major=True,
                                                                      beta=beta),
                                value=None if getattr(param, "main_grad", None) is not None else
                                gemm(lhs, rhs, out_dtype=param.dtype, a_mn_major=True, b_mn_major=True))

        def bias_grad(param: torch.Tensor | None, g: torch.Tensor) -> torch.Tensor | None:
            if param is None:
                return None
            return deliver_grad(param, compute=lambda out, beta: _column_sum(g, out, beta),
                                value=None if getattr(param, "main_grad", None) is not None else _column_sum(g).to(param.dtype))

        dw2 = weight_grad(w2, dy2, a) if ctx.needs_input_grad[3] else None
        db2 = bias_grad(b2, dy2) if ctx.needs_input_grad[4] else None
        dx = gemm(dh, w1c, b_mn_major=True).view(*dy.shape[:-1], w1c.shape[1]) if ctx.needs_input_grad[0] else None
        dw1 = weight_grad(w1, dh, x2) if ctx.needs_input_grad[1] else None
        db1 = bias_grad(b1, dh) if ctx.needs_input_grad[2] else None
        return dx, dw1, db1, dw2, db2


def swiglu_mlp_supported(ffn_features: int) -> bool:
    """Whether :func:`swiglu_mlp` runs fused on CUDA for ``ffn_features`` (F) gate / up features."""
    return ffn_features > 0 and ffn_features % 128 == 0


def swiglu_mlp(x: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor | None, w2: torch.Tensor, b2: torch.Tensor | None) -> torch.Tensor:
    """``(silu(gate) * up) w2^T + b2`` with ``[gate | up] = x w1^T + b1``; both SwiGLU passes in GEMM epilogues on CUDA."""
    if not x.is_cuda:
        h = F.linear(x, w1.to(x.dtype), None if b1 is None else b1.to(x.dtype))
        return F.linear(swiglu(h), w2.to(x.dtype), None if b2 is None else b2.to(x.dtype))
    return _SwiGLUMLPFunction.apply(x, w1, b1, w2, b2)


def swiglu(h: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` for ``h = [gate | up]`` along the last dimension."""
    if not h.is_cuda:
        gate, up = h.chunk(2, dim=-1)
        return (F.silu(gate.float()) * up.float()).to(h.dtype)
    return _SwiGLUFunction.apply(h)
