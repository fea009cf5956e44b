"""Component tier: loss scaling, data sampling, gradient-norm weighting, RNG streams, width-1 TP layers and
causal attention masking (reference ``tests/unit/test_single_process_components.py``)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from hybrid_training.distributed import launch_workers
from hybrid_training.distributed.groups import GroupHandle

from . import component_workers as C


@pytest.mark.distributed
def test_loss_scaler_skips_and_backs_off_on_every_rank() -> None:
    results = launch_workers(C.scaler_vote_worker, 2, timeout_seconds=180)
    traces = [r.value["trace"] for r in results]
    assert traces[0] == traces[1], "the overflow vote must give every rank the same decision"
    t = traces[0]
    assert t[0] == {"skipped": True, "scale": 512.0, "moved": False}
    assert not t[1]["skipped"] and t[1]["moved"] and t[1]["scale"] == 512.0
    assert t[2]["scale"] == 1024.0  # growth after growth_interval=2 clean steps
    assert results[0].value["state"]["skipped_steps"] == 1


@pytest.mark.distributed
@pytest.mark.parametrize("world", [2, 4])
def test_distributed_gradient_norm_counts_each_element_once(world: int) -> None:
    for r in launch_workers(C.tp_grad_norm_worker, world, timeout_seconds=180):
        assert abs(r.value["norm"] - r.value["expect"]) < 1e-9 * max(1.0, r.value["expect"])


def test_sampler_gives_tensor_peers_the_same_batches() -> None:
    from hybrid_training.training.data import DistributedBatchSampler

    def indices(local: int, size: int) -> list:
        group = GroupHandle(name="dp_shard", ranks=tuple(range(size)), local_rank=local, global_rank=local, process_group=None)
        return list(DistributedBatchSampler(64, 4, group, shuffle=True, seed=3).iter_epoch(1))

    a, b = indices(0, 2), indices(1, 2)
    assert len(a) == len(b) == 8
    flat_a = {i for batch in a for i in batch}
    flat_b = {i for batch in b for i in batch}
    assert not flat_a & flat_b and len(flat_a | flat_b) == 64  # data ranks partition the epoch
    assert indices(0, 2) == a  # deterministic for the same (seed, epoch)
    assert DistributedBatchSampler(64, 4, GroupHandle.trivial("dp_shard"), shuffle=True, seed=3).epoch_order(1).tolist() != \
        DistributedBatchSampler(64, 4, GroupHandle.trivial("dp_shard"), shuffle=True, seed=3).epoch_order(2).tolist()


def test_rng_capture_restore_and_temporary_seed() -> None:
    from hybrid_training.utils.reproducibility import (
        capture_rng_state,
        restore_rng_state,
        rng_state_from_serialisable,
        rng_state_to_serialisable,
        temporary_seed,
    )

    torch.manual_seed(5)
    snap = capture_rng_state(include_cuda=False)
    first = torch.rand(4)
    restore_rng_state(rng_state_from_serialisable(rng_state_to_serialisable(snap)))
    assert torch.equal(torch.rand(4), first)
    outer = torch.rand(2)
    torch.manual_seed(5)
    torch.rand(4)
    with temporary_seed(123):
        inner = torch.rand(3)
    assert torch.equal(torch.rand(2), outer), "temporary_seed must restore the surrounding stream"
    with temporary_seed(123):
        assert torch.equal(torch.rand(3), inner)


def test_width_one_parallel_layers_equal_plain_layers() -> None:
    from hybrid_training.models.transformer import build_reference_linear
    from hybrid_training.parallel import ColumnParallelLinear, RowParallelLinear

    g = GroupHandle.trivial("tensor")
    x = torch.randn(5, 12)
    ref = build_reference_linear(12, 6, bias=True, init_seed=4)
    col = ColumnParallelLinear(12, 6, g, bias=True, init_seed=4)
    row = RowParallelLinear(12, 6, g, bias=True, init_seed=4)
    assert torch.equal(col(x), ref(x)) and torch.allclose(row(x), ref(x), atol=1e-6)


def test_causal_attention_ignores_future_tokens() -> None:
    from hybrid_training.ops import reference_attention

    torch.manual_seed(0)
    b, s, h, d = 2, 7, 2, 8
    qkv = torch.randn(b, s, 3 * h * d)
    out = reference_attention(qkv, h, h, d, causal=True)
    changed = qkv.clone()
    changed[:, 4:] += torch.randn_like(changed[:, 4:])  # perturb tokens 4.. only
    out2 = reference_attention(changed, h, h, d, causal=True)
    assert torch.allclose(out[:, :4], out2[:, :4], atol=1e-6)
    assert not torch.allclose(out[:, 4:], out2[:, 4:])
    q, k, v = qkv.view(b, s, 3, h, d).unbind(2)
    expect = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
    assert torch.allclose(out.view(b, s, h, d), expect.transpose(1, 2), atol=1e-5)


def test_trace_ranges_are_inert_without_a_gpu_and_toggle() -> None:
    from hybrid_training.utils.tracing import set_tracing, trace_range, tracing_enabled

    set_tracing(True)
    try:
        with trace_range("test/range"):
            x = torch.ones(2) + 1
        assert torch.equal(x, torch.full((2,), 2.0))
        assert tracing_enabled() == torch.cuda.is_available()
    finally:
        set_tracing(False)
    assert not tracing_enabled()


@pytest.mark.parametrize(("sizes", "mode", "expect_ops"), [
    (dict(data_parallel_size=8), "disabled", {("backward", "data_parallel")}),
    (dict(shard_parallel_size=2, data_parallel_size=2), "disabled", {("backward", "shard"), ("backward", "data_parallel")}),
    (dict(data_parallel_size=2, tensor_parallel_size=4), "tensor_group", {("forward", "tensor"), ("backward", "tensor"),
                                                                         ("backward", "data_parallel")}),
])
def test_parallel_plan_names_each_collective_and_its_implementation(sizes: dict, mode: str, expect_ops: set) -> None:
    from types import SimpleNamespace

    from hybrid_training.config import ExperimentConfig, TopologyConfig
    from hybrid_training.distributed.topology import ParallelTopology
    from hybrid_training.parallel import describe_parallel_plan

    topo_cfg = TopologyConfig(sequence_parallel_mode=mode, **sizes)
    cfg = ExperimentConfig(topology=topo_cfg)
    world = 1
    for v in sizes.values():
        world *= v
    for device, library in ((torch.device("cpu"), "Gloo"), (torch.device("cuda"), "NCCL")):
        ctx = SimpleNamespace(topology=ParallelTopology(topo_cfg, world), device=device)
        plan = describe_parallel_plan(cfg, ctx)
        seen = {(s.phase, s.group) for s in plan.steps}
        want = set(expect_ops)
        if device.type == "cuda" and sizes.get("shard_parallel_size", 1) > 1 and sizes.get("data_parallel_size", 1) > 1:
            # hybrid sharding on CUDA: one fused kernel sums every replica's slice over the replicas x shards
            want = {("backward", "dp_shard")} | {op for op in want if op[1] not in ("shard", "data_parallel")}
        assert want <= seen, (want, seen)
        text = plan.render()
        assert plan.strategy in text and "metrics:" in text
        for s in plan.steps:
            assert s.implementation and s.operation in text
        if device.type == "cpu":
            assert all("kernel" not in s.implementation or library in s.implementation for s in plan.steps
                       if s.group == "data_parallel"), "no in-kernel collective is claimed on CPU"
        elif sizes.get("shard_parallel_size", 1) == 1 and "data_parallel_size" in sizes:
            dp_step = next(s for s in plan.steps if s.group == "data_parallel")
            assert "in-kernel NVLink" in dp_step.implementation
