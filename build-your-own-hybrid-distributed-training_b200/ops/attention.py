"""Causal flash attention over a packed QKV tensor, with GQA, plus RoPE.

``attention(qkv, num_heads, num_kv_heads, head_dim)`` takes the QKV projection
output as produced by the fused QKV GEMM -- ``[B, S, (H + 2*Hkv) * D]`` with the
``H`` query heads first, then the key heads, then the value heads -- and
returns ``[B, S, H * D]``, the layout the output projection consumes, so no
transpose or split is ever materialised.  The score matrix is never stored:
the forward keeps the per-row log-sum-exp and the backward recomputes the
probabilities (``csrc/attention.cu``).  This replaces the reference's
explicit ``(B, h, S, S)`` softmax (``src/hybrid_training/models/transformer.py:253-295``).

``apply_rope`` rotates the query and key heads of the packed tensor in place
of a copy (rotate-half convention, as in Llama); its backward applies the
inverse rotation.
"""

from __future__ import annotations

import math
from typing import Any

import torch

from ._ext import extension

__all__ = ["apply_rope", "attention", "reference_attention", "rope_tables"]


def rope_tables(seq_len: int, head_dim: int, theta: float, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """``cos``/``sin`` tables of shape ``[seq_len, head_dim // 2]`` (fp32)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    angles = torch.outer(torch.arange(seq_len, dtype=torch.float64), inv)
    return angles.cos().float().to(device), angles.sin().float().to(device)


def _split(qkv: torch.Tensor, h: int, hkv: int, d: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    b, s, _ = qkv.shape
    q = qkv[..., : h * d].reshape(b, s, h, d)
    k = qkv[..., h * d: (h + hkv) * d].reshape(b, s, hkv, d)
    v = qkv[..., (h + hkv) * d:].reshape(b, s, hkv, d)
    return q, k, v


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, inverse: bool = False) -> torch.Tensor:
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    c = cos[None, : x.shape[1], None, :]
    s = sin[None, : x.shape[1], None, :]
    if inverse:
        s = -s
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


def reference_attention(qkv: torch.Tensor, num_heads: int, num_kv_heads: int, head_dim: int, *, causal: bool = True) -> torch.Tensor:
    """Explicit fp32 softmax attention (the oracle and the CPU path)."""
    q, k, v = _split(qkv, num_heads, num_kv_heads, head_dim)
    groups = num_heads // num_kv_heads
    qf = q.float().transpose(1, 2)
    kf = k.float().transpose(1, 2).repeat_interleave(groups, dim=1)
    vf = v.float().transpose(1, 2).repeat_interleave(groups, dim=1)
    scores = qf @ kf.transpose(-1, -2) / math.sqrt(head_dim)
    if causal:
        s = scores.shape[-1]
        mask = torch.ones(s, s, dtype=torch.bool, device=qkv.device).triu(1)
        scores = scores.masked_fill(mask, float("-inf"))
    out = torch.softmax(scores, dim=-1) @ vf
    b, _, s, _ = out.shape
    return out.transpose(1, 2).reshape(b, s, num_heads * head_dim).to(qkv.dtype)


class _AttentionFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, qkv: torch.Tensor, h: int, hkv: int, d: int, causal: bool) -> torch.Tensor:
        b, s, _ = qkv.shape
        qkv = qkv.contiguous()
        out = torch.empty(b, s, h * d, dtype=qkv.dtype, device=qkv.device)
        lse = torch.empty(b, h, s, dtype=torch.float32, device=qkv.device)
        extension().attention_forward(qkv, out, lse, h, hkv, d, bool(causal), 1.0 / math.sqrt(d))
        ctx.save_for_backward(qkv, out, lse)
        ctx.dims = (h, hkv, d, causal)
        return out

    @staticmethod
    def backward(ctx: Any, dout: torch.Tensor) -> tuple[Any, ...]:
        qkv, out, lse = ctx.saved_tensors
        h, hkv, d, causal = ctx.dims
        b, s, _ = qkv.shape
        dqkv = torch.empty_like(qkv)
        delta = torch.empty(b, h, s, dtype=torch.float32, device=qkv.device)
        extension().attention_backward(qkv, out, dout.contiguous(), lse, delta, dqkv, h, hkv, d, bool(causal),
                                       1.0 / math.sqrt(d))
        return dqkv, None, None, None, None


def attention_window_forward(full: torch.Tensor, h: int, hkv: int, d: int, q_begin: int, q_len: int,
                             causal: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Attention of the queries ``[q_begin, q_begin + q_len)`` of a packed ``full`` tensor against all its keys.

    Returns ``(out_full, lse)``: ``out_full`` is ``[B, S, H*D]`` with the window's rows written and
    every other row zero; ``lse`` is ``[B, H, S]`` (meaningful inside the window).  The query
    columns of ``full`` outside the window are never read.  ``q_begin`` is a multiple of 128.
    """
    b, s, _ = full.shape
    out = torch.zeros(b, s, h * d, dtype=full.dtype, device=full.device)
    lse = torch.empty(b, h, s, dtype=torch.float32, device=full.device)
    extension().attention_forward(full, out, lse, h, hkv, d, bool(causal), 1.0 / math.sqrt(d), int(q_begin), int(q_len))
    return out, lse


def attention_window_backward(full: torch.Tensor, out: torch.Tensor, lse: torch.Tensor, dout_window: torch.Tensor, h: int,
                              hkv: int, d: int, q_begin: int, q_len: int, causal: bool) -> torch.Tensor:
    """Gradient of :func:`attention_window_forward`: ``dqkv`` ``[B, S, W]`` with dQ in the window's rows and
    dK / dV for every key (summed over the window's queries).  dQ rows outside the window are undefined."""
    b, s, _ = full.shape
    dout = torch.zeros(b, s, h * d, dtype=full.dtype, device=full.device)
    dout[:, q_begin:q_begin + q_len] = dout_window
    dqkv = torch.empty_like(full)
    delta = torch.empty(b, h, s, dtype=torch.float32, device=full.device)
    extension().attention_backward(full, out, dout, lse, delta, dqkv, h, hkv, d, bool(causal), 1.0 / math.sqrt(d),
                                   int(q_begin), int(q_len))
    return dqkv


def attention(qkv: torch.Tensor, num_heads: int, num_kv_heads: int, head_dim: int, *, causal: bool = True) -> torch.Tensor:
    """Attention over a packed ``[B, S, (H + 2*Hkv) * D]`` tensor; returns ``[B, S, H*D]``."""
    if not qkv.is_cuda:
        return reference_attention(qkv, num_heads, num_kv_heads, head_dim, causal=causal)
    return _AttentionFunction.apply(qkv, num_heads, num_kv_heads, head_dim, causal)


class _RopeFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rotated_heads: int, d: int) -> torch.Tensor:
        out = qkv.contiguous().clone()
        extension().rope_(out, cos, sin, rotated_heads, d, False)
        ctx.save_for_backward(cos, sin)
        ctx.dims = (rotated_heads, d)
        return out

    @staticmethod
    def backward(ctx: Any, grad: torch.Tensor) -> tuple[Any, ...]:
        cos, sin = ctx.saved_tensors
        g = grad.contiguous().clone()
        extension().rope_(g, cos, sin, ctx.dims[0], ctx.dims[1], True)
        return g, None, None, None, None


def apply_rope(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, num_heads: int, num_kv_heads: int,
               head_dim: int) -> torch.Tensor:
    """Rotate the query and key heads of a packed QKV tensor (values untouched)."""
    rotated = num_heads + num_kv_heads
    if not qkv.is_cuda:
        b, s, _ = qkv.shape
        qk = qkv[..., : rotated * head_dim].reshape(b, s, rotated, head_dim)
        qk = _rotate(qk, cos, sin).reshape(b, s, rotated * head_dim)
        return torch.cat([qk, qkv[..., rotated * head_dim:]], dim=-1)
    return _RopeFunction.apply(qkv, cos, sin, rotated, head_dim)
