"""Output head + (vocab-parallel) cross-entropy as one autograd op.

``lm_head_cross_entropy(h, weight, targets, group)`` computes
``mean_t CE(h_t @ W^T, target_t)`` where ``W`` is this rank's slice of the
vocabulary (rows ``[vocab_start, vocab_start + V/T)``).  Instead of gathering
the full ``(tokens, V)`` logits on every rank -- what the reference does with
``gather_output=True`` (``src/hybrid_training/models/transformer.py:502-512``)
-- each rank computes, per token, its local max, its local sum of
exponentials and (if it owns the target) the target logit; the ranks exchange
those three floats per token, form the global log-sum-exp, and each rank
writes the gradient of its own logit slice.  With one rank the whole
computation is a single kernel that reads each logit row once and writes its
gradient (``csrc/cross_entropy.cu``).

The gradient of the logits is produced during the forward pass (it is needed
anyway and the logits are then dead); the backward pass feeds it to the dgrad
and wgrad GEMMs with the incoming loss gradient as a device-side scale, so no
host synchronisation is needed and the step can be captured in a CUDA graph.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.nn.functional as F

from ..distributed.collectives import all_gather_tensor
from ..distributed.groups import GroupHandle
from ._ext import extension
from .grads import deliver_grad
from .linear import compute_weight, gemm

__all__ = ["cross_entropy", "lm_head_cross_entropy", "reference_vocab_parallel_cross_entropy"]

_VOCAB_PAD = 64


def reference_vocab_parallel_cross_entropy(local_logits: torch.Tensor, targets: torch.Tensor, vocab_start: int,
                                           group: GroupHandle | None) -> torch.Tensor:
    """Differentiable vocab-parallel CE in plain PyTorch (CPU path / oracle); returns the mean loss."""
    from ..autograd.collectives import all_gather_along_dim

    logits = local_logits.float().reshape(-1, local_logits.shape[-1])
    t = targets.reshape(-1)
    if group is None or group.is_trivial:
        return F.cross_entropy(logits, t)
    vl = logits.shape[-1]
    local_max = logits.detach().max(-1, keepdim=True).values
    global_max = all_gather_along_dim(local_max, group, -1).max(-1, keepdim=True).values
    shifted = logits - global_max
    sum_exp = shifted.exp().sum(-1, keepdim=True)
    owned = (t >= vocab_start) & (t < vocab_start + vl)
    idx = (t - vocab_start).clamp(0, vl - 1)
    target_logit = shifted.gather(-1, idx[:, None]) * owned[:, None]
    from ..autograd.collectives import reduce_from_group

    total_exp = reduce_from_group(sum_exp, group)
    total_target = reduce_from_group(target_logit, group)
    return (total_exp.log() - total_target).mean()


class _HeadCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, h: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor, group: GroupHandle | None,
                vocab_start: int, vocab_size: int) -> torch.Tensor:
        ext = extension()
        h2 = h.reshape(-1, h.shape[-1]).contiguous()
        t = targets.reshape(-1).contiguous()
        rows = h2.shape[0]
        w = compute_weight(weight, h.dtype)
        vl = w.shape[0]
        padded = -(-vl // _VOCAB_PAD) * _VOCAB_PAD
        storage = torch.empty(rows, padded, dtype=h.dtype, device=h.device)
        logits = storage[:, :vl]
        gemm(h2, w, out=logits)
        loss = torch.zeros(1, dtype=torch.float32, device=h.device)
        scale = 1.0 / rows
        if group is None or group.is_trivial:
            ext.cross_entropy_fused(logits, t, logits, loss, vocab_start, scale)
        else:
            stats = torch.empty(rows, 3, dtype=torch.float32, device=h.device)
            ext.cross_entropy_stats(logits, t, stats, vocab_start)
            gathered, work = all_gather_tensor(stats, group)
            work.wait()
            lse = torch.empty(rows, dtype=torch.float32, device=h.device)
            ext.cross_entropy_combine(gathered, lse, loss, group.size, scale)
            ext.cross_entropy_grad(logits, t, lse, logits, vocab_start, scale)
        # ``logits`` now holds d(loss)/d(logits) for a unit incoming gradient.
        ctx.save_for_backward(h2, w, storage)
        ctx.vl, ctx.shape, ctx.weight = vl, h.shape, weight
        return loss[0]

    @staticmethod
    def backward(ctx: Any, grad: torch.Tensor) -> tuple[Any, ...]:
        h2, w, storage = ctx.saved_tensors
        dlogits = storage[:, : ctx.vl]
        alpha = grad.reshape(1).float().contiguous()
        dh = None
        if ctx.needs_input_grad[0]:
            dh = gemm(dlogits, w, b_mn_major=True, alpha=alpha).view(ctx.shape)
        dw = None
        if ctx.needs_input_grad[1]:
            weight = ctx.weight
            dw = deliver_grad(weight, compute=lambda out, beta: gemm(dlogits, h2, out=out, a_mn_major=True, b_mn_major=True,
                                                                      beta=beta, alpha=alpha),
                              value=None if getattr(weight, "main_grad", None) is not None else
                              gemm(dlogits, h2, out_dtype=weight.dtype, a_mn_major=True, b_mn_major=True, alpha=alpha))
        return dh, dw, None, None, None, None


def lm_head_cross_entropy(h: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor, *,
                          group: GroupHandle | None = None, vocab_start: int = 0, vocab_size: int | None = None) -> torch.Tensor:
    """Mean next-token CE of ``h @ weight^T`` against ``targets`` with a vocab-sharded ``weight``."""
    if not h.is_cuda:
        logits = F.linear(h, weight.to(h.dtype))
        return reference_vocab_parallel_cross_entropy(logits, targets, vocab_start, group)
    return _HeadCrossEntropy.apply(h, weight, targets, group, vocab_start, vocab_size or weight.shape[0])


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Mean CE over the last dimension (reference ``engine.py:102-112`` semantics)."""
    return F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), targets.reshape(-1))
