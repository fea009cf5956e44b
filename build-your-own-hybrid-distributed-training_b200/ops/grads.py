"""Gradient delivery into flat ``main_grad`` buffers.

A parameter may carry ``main_grad``: an fp32 view into a flat gradient buffer
owned by DDP (one bucket per slice), FSDP or the optimizer.  The native
backward kernels then write the weight gradient straight into that view (the
wgrad GEMM epilogue overwrites on the first micro-batch of a step and
accumulates afterwards) and call ``param.grad_ready_hook(param)``, which is how
DDP learns that a bucket slot is filled.  Parameters without ``main_grad`` get
an ordinary autograd gradient.  This replaces the reference's
copy-into-bucket step (``src/hybrid_training/parallel/ddp.py:513``).
"""

from __future__ import annotations

from collections.abc import Callable

import torch

__all__ = ["adopt_exposed_gradient", "deliver_grad", "has_main_grad", "main_grad_beta", "reset_main_grad_state"]


def has_main_grad(param: torch.Tensor | None) -> bool:
    return param is not None and getattr(param, "main_grad", None) is not None


def adopt_exposed_gradient(param: torch.Tensor, *, from_autograd: bool) -> None:
    """Decide how the first delivery after a synchronisation writes ``main_grad``.

    After a step, data parallelism exposes ``param.grad`` as a view of ``main_grad``
    (``_grad_exposed``).  If the caller released it (``zero_grad(set_to_none=True)``)
    the next delivery overwrites; if the caller kept it (zeroed in place, or left it to
    accumulate across steps as plain PyTorch allows) a native delivery accumulates onto
    it.  A gradient that reaches us through autograd already contains the kept value
    (autograd accumulated into ``param.grad``), so it always overwrites.
    """
    if getattr(param, "_grad_exposed", False):
        param._grad_exposed = False
        if from_autograd or param.grad is None:
            param.main_grad_fresh = True


def main_grad_beta(param: torch.Tensor) -> float:
    """0.0 for the first write of a step (overwrite), 1.0 afterwards (accumulate)."""
    return 0.0 if getattr(param, "main_grad_fresh", True) else 1.0


def deliver_grad(param: torch.Tensor, compute: Callable[[torch.Tensor, float], None] | None = None,
                 value: torch.Tensor | None = None, *, native: bool = True) -> torch.Tensor | None:
    """Write a weight gradient into ``param.main_grad`` (or return ``value`` for autograd).

    ``compute(out, beta)`` must write ``out = grad + beta * out``; when it is
    not given, ``value`` is copied or added.  A parameter used by several native
    ops in one backward (a tied embedding/head weight) declares the count in
    ``param.native_grad_uses``; ``grad_ready_hook`` then runs after the last of
    those deliveries.  Deliveries of autograd-accumulated gradients
    (``native=False``) already hold every contribution.
    """
    main = getattr(param, "main_grad", None)
    if main is None:
        if value is None:
            raise ValueError("deliver_grad needs a value when the parameter has no main_grad")
        return value
    adopt_exposed_gradient(param, from_autograd=not native)
    beta = main_grad_beta(param)
    if compute is not None:
        compute(main, beta)
    elif beta == 0.0:
        main.copy_(value.reshape(main.shape))
    else:
        main.add_(value.reshape(main.shape))
    param.main_grad_fresh = False
    uses = getattr(param, "native_grad_uses", 1) if native else 1
    if uses > 1:
        seen = getattr(param, "_native_deliveries", 0) + 1
        if seen < uses:
            param._native_deliveries = seen
            return None
        param._native_deliveries = 0
    hook = getattr(param, "grad_ready_hook", None)
    if hook is not None:
        hook(param)
    return None


def reset_main_grad_state(params: list[torch.Tensor]) -> None:
    """Mark every ``main_grad`` as stale so the next delivery overwrites it."""
    for p in params:
        if getattr(p, "main_grad", None) is not None:
            p.main_grad_fresh = True
        if getattr(p, "_native_deliveries", 0):
            p._native_deliveries = 0
