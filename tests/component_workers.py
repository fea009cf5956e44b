"""Gloo workers for the component tests: loss-scaler overflow vote, distributed gradient norm under TP."""

from __future__ import annotations

from typing import Any

import torch
import torch.nn as nn

from hybrid_training.config import GradScalerConfig, TopologyConfig
from hybrid_training.distributed import init_distributed


def scaler_vote_worker(rank: int, world: int) -> dict[str, Any]:
    """Rank 1 produces a non-finite gradient: every rank must skip the step and back off together."""
    from hybrid_training.optim.grad_scaler import GradScaler

    ctx = init_distributed(TopologyConfig(data_parallel_size=world), backend="gloo", device="cpu")
    try:
        cfg = GradScalerConfig(enabled=True, init_scale=1024.0, growth_interval=2)
        scaler = GradScaler(cfg, ctx.group("world"), torch.device("cpu"))
        p = nn.Parameter(torch.ones(3))
        opt = torch.optim.SGD([p], lr=1.0)
        trace = []
        for step in range(4):
            p.grad = torch.full((3,), 1024.0)
            if step == 0 and rank == 1:
                p.grad[1] = float("inf")
            before = p.detach().clone()
            scaler.step(opt, [p])
            scale = scaler.update()
            trace.append({"skipped": scaler.last_step_skipped, "scale": scale, "moved": not torch.equal(before, p.detach())})
        return {"trace": trace, "state": scaler.state_dict()}
    finally:
        ctx.shutdown()


def tp_grad_norm_worker(rank: int, world: int) -> dict[str, float]:
    """Weighted distributed norm of a TP-partitioned + replicated parameter set equals the full norm."""
    from hybrid_training.optim.sharded_optimizer import build_gradient_norm_contributions, distributed_gradient_norm

    ctx = init_distributed(TopologyConfig(tensor_parallel_size=world), backend="gloo", device="cpu")
    try:
        g = ctx.group("tensor")
        full_w = torch.arange(8 * world, dtype=torch.float32).reshape(4 * world, 2) / 7
        bias = torch.tensor([0.5, -1.5])  # replicated: same gradient on every rank
        w = nn.Parameter(torch.zeros(4, 2))
        w.grad = full_w[rank * 4:(rank + 1) * 4].clone()
        w.is_tensor_parallel_replicated = False
        w.tensor_parallel_group_size = world
        b = nn.Parameter(torch.zeros(2))
        b.grad = bias.clone()
        contributions = build_gradient_norm_contributions([w, b], world_size=world)
        norm = float(distributed_gradient_norm(contributions, g, device=torch.device("cpu")))
        expect = float(torch.sqrt(full_w.double().square().sum() + bias.double().square().sum()))
        return {"norm": norm, "expect": expect}
    finally:
        ctx.shutdown()
