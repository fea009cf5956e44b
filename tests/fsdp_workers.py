"""Workers for the FSDP feature tests (run in ranks spawned by ``launch_workers`` on CPU/Gloo)."""

from __future__ import annotations

from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from hybrid_training.config import FSDPConfig, TopologyConfig
from hybrid_training.distributed import init_distributed
from hybrid_training.errors import HybridTrainingError
from hybrid_training.models import MLP
from hybrid_training.parallel import FullyShardedDataParallel

from .dist_workers import MLP_CFG, mlp_batch


def _ctx(world: int):
    return init_distributed(TopologyConfig(shard_parallel_size=world), backend="gloo", device="cpu")


def summon_worker(rank: int, world: int) -> dict[str, Any]:
    """Full parameters inside summon_full_params; edits persist only with writeback; nothing stays gathered."""
    ctx = _ctx(world)
    try:
        names = [n for n, _ in MLP(MLP_CFG, seed=0).named_parameters()]
        fsdp = FullyShardedDataParallel(MLP(MLP_CFG, seed=0), ctx.group("shard"))

        def attr(path: str) -> torch.Tensor:
            obj: Any = fsdp.module
            for part in path.split("."):
                obj = obj[int(part)] if part.isdigit() else getattr(obj, part)
            return obj

        seen = {}
        with fsdp.summon_full_params():
            for name in names:
                seen[name] = attr(name).detach().clone()
            attr("head.weight").fill_(123.0)  # discarded: no writeback
        after_plain = fsdp.full_state_dict()
        held_between = fsdp.memory_summary()["full_bytes"]
        with fsdp.summon_full_params(writeback=True):
            for name in names:
                attr(name).mul_(2.0)
        after_writeback = fsdp.full_state_dict()
        return {"seen": seen, "after_plain": after_plain, "after_writeback": after_writeback, "held_between": held_between,
                "held_after": fsdp.memory_summary()["full_bytes"]}
    finally:
        ctx.shutdown()


def no_sync_worker(rank: int, world: int, micro: int) -> dict[str, Any]:
    """Gradient after ``micro`` micro-batches (all but the last under no_sync) and one reduction."""
    ctx = _ctx(world)
    try:
        fsdp = FullyShardedDataParallel(MLP(MLP_CFG, seed=0), ctx.group("shard"), FSDPConfig(check_reduction_order=True))
        for i in range(micro):
            x, y = mlp_batch(i, rank)
            cm = fsdp.no_sync() if i < micro - 1 else _null()
            with cm:
                (F.mse_loss(fsdp(x), y) / micro).backward()
        fsdp.finish_backward()
        return {"grad": fsdp.handle.flat_param.grad.detach().clone(), "range": (fsdp.handle.local_shard_range().start,
                                                                                   fsdp.handle.shard_numel),
                "reductions": fsdp.handle.reduction_count}
    finally:
        ctx.shutdown()


class _null:
    def __enter__(self) -> None:
        return None

    def __exit__(self, *a: object) -> None:
        return None


def offload_worker(rank: int, world: int, offload: bool, steps: int) -> dict[str, Any]:
    """A few AdamW steps with the master shard in host memory (or not); returns the full parameters."""
    from hybrid_training.optim import FusedAdamW

    ctx = _ctx(world)
    try:
        fsdp = FullyShardedDataParallel(MLP(MLP_CFG, seed=0), ctx.group("shard"), FSDPConfig(cpu_offload_params=offload))
        opt = FusedAdamW([fsdp.handle.flat_param], lr=1e-3, weight_decay=0.0)
        for step in range(steps):
            x, y = mlp_batch(step, rank)
            F.mse_loss(fsdp(x), y).backward()
            fsdp.finish_backward()
            opt.step()
            opt.zero_grad()
        return {"full": fsdp.full_state_dict(), "device": str(fsdp.handle.flat_param.device)}
    finally:
        ctx.shutdown()


def auto_wrap_worker(rank: int, world: int, threshold: int, steps: int) -> dict[str, Any]:
    """Units created by the auto-wrap threshold, their sizes, and the parameters after training."""
    from hybrid_training.optim import FusedAdamW

    ctx = _ctx(world)
    try:
        fsdp = FullyShardedDataParallel(MLP(MLP_CFG, seed=0), ctx.group("shard"), FSDPConfig(auto_wrap_min_num_params=threshold))
        units = [u for u in fsdp.fsdp_units() if u.handle is not None]
        sizes = sorted(u.handle.total_numel for u in units)
        opt = FusedAdamW([u.handle.flat_param for u in units], lr=1e-3, weight_decay=0.0)
        for step in range(steps):
            x, y = mlp_batch(step, rank)
            F.mse_loss(fsdp(x), y).backward()
            fsdp.finish_backward()
            opt.step()
            opt.zero_grad()
        return {"units": len(units), "sizes": sizes, "full": fsdp.full_state_dict(),
                "padding_grad_zero": all(_padding_grad_is_zero(u) for u in units)}
    finally:
        ctx.shutdown()


def _padding_grad_is_zero(unit: FullyShardedDataParallel) -> bool:
    h = unit.handle
    g = h.flat_param.grad
    if g is None or not h.padding:
        return True
    r = h.local_shard_range()
    pad_start = h.total_numel
    lo = max(pad_start, r.start) - r.start
    return bool((g[lo:] == 0).all()) if lo < h.shard_numel else True


class _TiedPair(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.a = nn.Sequential(nn.Linear(8, 64), nn.ReLU())
        self.b = nn.Sequential(nn.Linear(64, 8))
        self.b[0].weight = nn.Parameter(self.a[0].weight.detach().t().contiguous())
        self.c = nn.Linear(8, 64)
        self.c.weight = self.a[0].weight  # shared between unit `a` and unit `c`

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.b(self.a(x)) + self.c(x).sum(-1, keepdim=True)


class _Frozen(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.a = nn.Linear(4, 4)
        self.b = nn.Linear(4, 4)
        self.b.weight.requires_grad_(False)


def rejection_worker(rank: int, world: int, case: str) -> str:
    """Construction-time refusals: cross-unit ties, mixed requires_grad, the gather limit, no parameters."""
    ctx = _ctx(world)
    try:
        group = ctx.group("shard")
        try:
            if case == "tied":
                FullyShardedDataParallel(_TiedPair(), group, FSDPConfig(auto_wrap_min_num_params=100))
            elif case == "frozen":
                FullyShardedDataParallel(_Frozen(), group)
            elif case == "limit":
                FullyShardedDataParallel(MLP(MLP_CFG, seed=0), group, FSDPConfig(limit_all_gather_bytes=64))
            elif case == "empty":
                FullyShardedDataParallel(nn.ReLU(), group)
            return "no error"
        except HybridTrainingError as exc:
            return type(exc).__name__ + ": " + str(exc)
    finally:
        ctx.shutdown()
