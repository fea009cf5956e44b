"""FSDP features beyond plain training, on CPU/Gloo ranks (reference ``tests/distributed/test_fsdp.py``).

summon_full_params (materialise, write back, free), no_sync accumulation with one reduction and the
reduction-order check on, CPU offload of the master shard, the auto-wrap threshold and nested units,
padding gradients, and the construction-time refusals (a parameter tied across units, mixed
requires_grad inside a unit, the all-gather size limit, a module without parameters).
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from hybrid_training.distributed import launch_workers
from hybrid_training.models import MLP

from . import dist_workers as W
from . import fsdp_workers as FW

pytestmark = pytest.mark.distributed


@pytest.mark.parametrize("world", [2, 4])
def test_summon_full_params_materialises_writes_back_and_frees(world: int) -> None:
    ref = dict(MLP(W.MLP_CFG, seed=0).named_parameters())
    for r in launch_workers(FW.summon_worker, world, timeout_seconds=300):
        v = r.value
        for name, p in ref.items():
            assert torch.equal(v["seen"][name], p.detach()), name  # every rank sees the full tensor
            assert torch.equal(v["after_plain"][name], p.detach()), name  # edits without writeback are dropped
            assert torch.equal(v["after_writeback"][name], 2 * p.detach()), name
        assert v["held_between"] == 0 and v["held_after"] == 0  # gathered buffers are freed on exit


@pytest.mark.parametrize("micro", [2, 3])
def test_no_sync_accumulation_matches_the_summed_loss_with_one_reduction(micro: int) -> None:
    world = 2
    model = MLP(W.MLP_CFG, seed=0)
    total = 0.0
    for i in range(micro):
        for r in range(world):
            x, y = W.mlp_batch(i, r)
            total = total + F.mse_loss(model(x), y) / (micro * world)
    total.backward()
    flat = torch.cat([p.grad.reshape(-1) for p in model.parameters()])
    for r in launch_workers(FW.no_sync_worker, world, args=(micro,), timeout_seconds=300):
        start, n = r.value["range"]
        expect = torch.zeros(n)
        valid = max(0, min(n, flat.numel() - start))
        expect[:valid] = flat[start:start + valid]
        assert torch.allclose(r.value["grad"], expect, atol=1e-6)
        assert r.value["reductions"] == 1  # accumulation costs one reduce-scatter, not `micro`


def test_cpu_offload_trains_like_the_resident_shard() -> None:
    on = launch_workers(FW.offload_worker, 2, args=(True, 3), timeout_seconds=300)
    off = launch_workers(FW.offload_worker, 2, args=(False, 3), timeout_seconds=300)
    assert on[0].value["device"] == "cpu"
    for name, t in off[0].value["full"].items():
        assert torch.allclose(on[0].value["full"][name], t, atol=1e-7), name


@pytest.mark.parametrize(("threshold", "units"), [(0, 1), (600, 2), (500, 3)])
def test_auto_wrap_threshold_nests_units_without_changing_results(threshold: int, units: int) -> None:
    steps = 3
    ref = W.single_process_mlp(2, steps=steps)
    results = launch_workers(FW.auto_wrap_worker, 2, args=(threshold, steps), timeout_seconds=300)
    v = results[0].value
    assert v["units"] == units, v["sizes"]
    assert sum(v["sizes"]) == sum(p.numel() for p in MLP(W.MLP_CFG, seed=0).parameters())
    assert all(r.value["padding_grad_zero"] for r in results)
    for name, p in ref["params"].items():
        assert torch.allclose(v["full"][name], p, atol=1e-5), name


@pytest.mark.parametrize(("case", "error"), [("tied", "UnsupportedFeatureError"), ("frozen", "UnsupportedFeatureError"),
                                             ("limit", "ShardingError"), ("empty", "ShardingError")])
def test_construction_refusals(case: str, error: str) -> None:
    for r in launch_workers(FW.rejection_worker, 2, args=(case,), timeout_seconds=300):
        assert r.value.startswith(error), r.value
        assert "Fix:" in r.value
