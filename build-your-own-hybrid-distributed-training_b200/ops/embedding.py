"""(Vocab-parallel) token embedding with an optional fused position table.

Rows outside ``[vocab_start, vocab_start + rows)`` produce zeros (another rank
owns them); the caller reduces over the tensor group, as in
``src/hybrid_training/parallel/tensor_parallel.py:575-590``.  The kernel
(``csrc/elementwise.cu``) gathers rows and adds the position row in one pass
and writes fp32, the dtype of the residual stream; the backward scatters the
incoming gradient into the fp32 ``main_grad`` of the table with atomics and
reduces the position gradient over the batch.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.nn.functional as F

from ._ext import extension
from .grads import deliver_grad

__all__ = ["embedding"]


class _EmbeddingFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, ids: torch.Tensor, weight: torch.Tensor, positions: torch.Tensor | None, vocab_start: int) -> torch.Tensor:
        b, s = ids.shape
        d = weight.shape[1]
        out = torch.empty(b, s, d, dtype=torch.float32, device=weight.device)
        ids32 = ids.to(torch.int32).contiguous()
        extension().embedding_forward(ids32, weight, positions, out, int(vocab_start))
        ctx.save_for_backward(ids32)
        ctx.weight, ctx.positions, ctx.vocab_start = weight, positions, vocab_start
        return out

    @staticmethod
    def backward(ctx: Any, grad: torch.Tensor) -> tuple[Any, ...]:
        (ids32,) = ctx.saved_tensors
        ext = extension()
        grad = grad.contiguous()
        weight, positions = ctx.weight, ctx.positions

        def scatter(out: torch.Tensor, beta: float) -> None:
            if beta == 0.0:
                out.zero_()
            ext.embedding_backward(ids32, grad, out, int(ctx.vocab_start))

        dw = None
        if ctx.needs_input_grad[1]:
            if getattr(weight, "main_grad", None) is not None:
                deliver_grad(weight, compute=scatter)
            else:
                dw = torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
                scatter(dw, 1.0)
                dw = dw.to(weight.dtype)
        dp = None
        if positions is not None and ctx.needs_input_grad[2]:
            s = grad.shape[1]

            def pos_grad(out: torch.Tensor, beta: float) -> None:
                if beta == 0.0 and out.shape[0] > s:
                    out[s:].zero_()
                ext.sum_batch_into(grad, out[:s], beta)

            if getattr(positions, "main_grad", None) is not None:
                deliver_grad(positions, compute=pos_grad)
            else:
                dp = torch.zeros(positions.shape, dtype=torch.float32, device=grad.device)
                pos_grad(dp, 0.0)
                dp = dp.to(positions.dtype)
        return None, dw, dp, None


def embedding(ids: torch.Tensor, weight: torch.Tensor, positions: torch.Tensor | None = None, *,
              vocab_start: int = 0) -> torch.Tensor:
    """``weight[ids - vocab_start]`` (zero outside this shard) ``+ positions[:S]``, as fp32 ``[B, S, d]``."""
    if not weight.is_cuda:
        rows = weight.shape[0]
        if vocab_start == 0 and rows > int(ids.max()):
            out = F.embedding(ids, weight)
        else:
            mask = (ids < vocab_start) | (ids >= vocab_start + rows)
            out = F.embedding((ids - vocab_start).clamp(0, rows - 1), weight).masked_fill(mask[..., None], 0.0)
        if positions is not None:
            out = out + positions[: ids.shape[1]][None]
        return out
    return _EmbeddingFunction.apply(ids, weight, positions, vocab_start)
