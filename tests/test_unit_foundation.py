"""Pure-function tests: config schema, topology arithmetic, flat layouts, errors, schedules, memory model."""

from __future__ import annotations

import dataclasses
import itertools
import math
from pathlib import Path

import pytest
import torch
import yaml

from hybrid_training.config import (
    DataConfig,
    ExperimentConfig,
    FSDPConfig,
    MixedPrecisionConfig,
    ModelConfig,
    SchedulerConfig,
    TopologyConfig,
    load_experiment_config,
    resolve_dtype,
)
from hybrid_training.distributed.topology import COMPOSITE_GROUPS, DIMENSIONS, ParallelTopology
from hybrid_training.errors import ConfigurationError, ShardingError, TopologyError, format_error
from hybrid_training.training.state import LearningRateSchedule, TrainingState
from hybrid_training.utils import (
    ShardRange,
    build_flat_layout,
    derive_seed,
    estimate_training_memory,
    even_shard_ranges,
    flatten_dense_tensors,
    intersect_ranges,
    pad_flat_tensor,
    split_tensor_along_dim,
    unflatten_to_views,
)

ROOT = Path(__file__).resolve().parent.parent


def test_format_error_has_five_parts() -> None:
    msg = format_error("op", "bad thing", rank=3, world_size=8, expected=1, observed=2, resolution="fix it")
    assert msg == "[rank 3/8] op: bad thing; expected 1, observed 2. Fix: fix it"


def test_config_rejects_unknown_keys_with_dotted_path() -> None:
    with pytest.raises(ConfigurationError, match="model.bogus"):
        ExperimentConfig.from_dict({"model": {"bogus": 1}})


def test_config_roundtrip_yaml(tmp_path: Path) -> None:
    cfg = ExperimentConfig(model=ModelConfig.llama_1b3(), topology=TopologyConfig(tensor_parallel_size=2,
                           sequence_parallel_mode="tensor_group"))
    path = cfg.to_yaml(tmp_path / "c.yaml")
    assert load_experiment_config(path) == cfg


@pytest.mark.parametrize("path", sorted((ROOT / "configs").glob("*.yaml")))
def test_shipped_configs_load(path: Path) -> None:
    cfg = load_experiment_config(path)
    assert cfg.topology.world_size >= 1


def test_reference_style_yaml_loads() -> None:
    raw = {"backend": "gloo", "device": "cpu", "topology": {"data_parallel_size": 2, "shard_parallel_size": 2,
                                                             "tensor_parallel_size": 2, "sequence_parallel_mode": "tensor_group"},
           "model": {"kind": "transformer", "hidden_size": 32, "num_heads": 4, "vocab_size": 64},
           "optimizer": {"betas": [0.9, 0.95]}, "tensor_parallel": {"sequence_parallel": True}}
    cfg = ExperimentConfig.from_dict(raw)
    assert cfg.optimizer.betas == (0.9, 0.95) and cfg.topology.world_size == 8


@pytest.mark.parametrize("bad", [dict(data_parallel_size=0), dict(sequence_parallel_size=2),
                                 dict(sequence_parallel_mode="tensor_group"), dict(sequence_parallel_mode="nope")])
def test_topology_config_validation(bad: dict) -> None:
    with pytest.raises(TopologyError):
        TopologyConfig(**bad)


def test_for_world_size_fills_first_missing_dimension() -> None:
    cfg = TopologyConfig.for_world_size(8, tensor_parallel_size=2)
    assert (cfg.data_parallel_size, cfg.tensor_parallel_size, cfg.world_size) == (4, 2, 8)
    with pytest.raises(TopologyError):
        TopologyConfig.for_world_size(6, tensor_parallel_size=4)


def test_mixed_precision_scaler_requires_fp16() -> None:
    with pytest.raises(ConfigurationError):
        MixedPrecisionConfig(enabled=True, param_dtype="bfloat16", scaler=dataclasses.replace(
            MixedPrecisionConfig().scaler, enabled=True))
    assert resolve_dtype("bf16") is torch.bfloat16


def test_fsdp_rejects_unpadded() -> None:
    with pytest.raises(ConfigurationError):
        FSDPConfig(use_padding=False)


def test_rank_grid_worked_example() -> None:
    topo = ParallelTopology(TopologyConfig(data_parallel_size=2, shard_parallel_size=2, tensor_parallel_size=2), 8)
    c = topo.coordinates_of(3)
    assert (c.data_parallel, c.shard, c.sequence, c.tensor) == (0, 1, 0, 1)
    assert topo.group_ranks("tensor", 3) == (2, 3)
    assert topo.group_ranks("shard", 3) == (1, 3)
    assert topo.group_ranks("data_parallel", 3) == (3, 7)
    assert topo.group_ranks("dp_shard", 3) == (1, 3, 5, 7)
    assert topo.neighbour_ranks("dp_shard", 3) == (1, 5)


def _factorisations(n: int):
    for dp, sh, sq, tp in itertools.product(range(1, n + 1), repeat=4):
        if dp * sh * sq * tp == n:
            yield dp, sh, sq, tp


@pytest.mark.parametrize("world", [1, 2, 3, 4, 6, 8])
def test_all_dimension_combinations_partition_the_world(world: int) -> None:
    for dp, sh, sq, tp in _factorisations(world):
        mode = "independent" if sq > 1 else "disabled"
        topo = ParallelTopology(TopologyConfig(dp, sh, sq, tp, mode), world)
        for r in range(world):
            assert topo.rank_of(topo.coordinates_of(r)) == r
        for name in (*DIMENSIONS, *COMPOSITE_GROUPS):
            groups = topo.all_group_rank_lists(name)
            flat = sorted(x for g in groups for x in g)
            assert flat == list(range(world)), (name, groups)
            assert all(len(g) == topo.size(name) for g in groups)


def test_flat_layout_and_views() -> None:
    a, b = torch.randn(3, 4), torch.randn(5)
    entries, total = build_flat_layout([("a", a), ("b", b)])
    assert total == 17 and entries[1].offset == 12
    flat = flatten_dense_tensors([a, b])
    va, vb = unflatten_to_views(flat, entries)
    assert torch.equal(va, a) and torch.equal(vb, b)
    with pytest.raises(ShardingError):
        build_flat_layout([("a", a), ("a", b)])


def test_padding_and_shard_ranges() -> None:
    padded = pad_flat_tensor(torch.ones(1633), 4)
    assert padded.numel() == 1636 and float(padded[-3:].sum()) == 0.0
    ranges = even_shard_ranges(1633, 4)
    assert [r.length for r in ranges] == [409] * 4 and ranges[-1].end == 1636
    assert intersect_ranges(ShardRange(0, 10), ShardRange(5, 10)) == ShardRange(5, 5)
    assert intersect_ranges(ShardRange(0, 5), ShardRange(5, 10)) is None


def test_split_tensor_along_dim_requires_divisibility() -> None:
    parts = split_tensor_along_dim(torch.arange(12).view(3, 4), 1, 2)
    assert parts[1].tolist() == [[2, 3], [6, 7], [10, 11]]
    with pytest.raises(ShardingError):
        split_tensor_along_dim(torch.arange(10), 0, 3)


def test_derive_seed_is_stable_and_stream_separated() -> None:
    assert derive_seed(0, "a", 1) == derive_seed(0, "a", 1)
    assert len({derive_seed(0, s, i) for s in "abc" for i in range(10)}) == 30
    assert 0 <= derive_seed(123, "x") < 2**31


@pytest.mark.parametrize("name", ["constant", "linear", "cosine"])
def test_lr_schedule_shapes(name: str) -> None:
    sched = LearningRateSchedule(SchedulerConfig(name=name, warmup_steps=4, min_lr_ratio=0.1), base_learning_rate=1.0,
                                 total_steps=20)
    assert sched.value_at(0) == pytest.approx(0.25)
    assert sched.value_at(3) == pytest.approx(1.0)
    end = sched.value_at(20)
    assert end == pytest.approx(1.0 if name == "constant" else 0.1)
    restored = LearningRateSchedule.from_state_dict(sched.state_dict())
    assert restored.value_at(11) == pytest.approx(sched.value_at(11))


def test_training_state_json_roundtrip() -> None:
    s = TrainingState(step=3, last_loss=float("nan"))
    d = s.as_dict()
    assert d["last_loss"] is None and d["best_eval_loss"] is None
    assert TrainingState.from_dict(d).step == 3


def test_memory_model_sharding() -> None:
    full = estimate_training_memory(1000, shard_group_size=1)
    sharded = estimate_training_memory(1000, shard_group_size=4, largest_unit_parameters=100)
    assert full.steady_state == 1000 * 16
    assert sharded.steady_state == 250 * 16 and sharded.transient_gathered_parameters == 400


def test_model_presets() -> None:
    g = ModelConfig.gpt2_124m()
    assert (g.hidden_size, g.num_layers, g.vocab_size, g.tie_word_embeddings) == (768, 12, 50257, True)
    l8 = ModelConfig.llama3_8b()
    assert l8.resolved_num_kv_heads == 8 and l8.head_dim == 128
    with pytest.raises(ConfigurationError):
        ModelConfig(kind="transformer", num_heads=4, num_kv_heads=3, hidden_size=32)
    with pytest.raises(ConfigurationError):
        DataConfig(token_distribution="zipf")
