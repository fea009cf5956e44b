"""Communication and memory accounting per step, asserted on counts and bytes, never on time.

Mirrors the reference's performance tier (``tests/performance/test_instrumentation.py``) for this
framework: every collective of one training step is counted with ``observe_collectives`` while the
engine runs on CPU/Gloo ranks.
"""

from __future__ import annotations

import pytest

from hybrid_training.distributed import launch_workers
from hybrid_training.models import MLP
from hybrid_training.utils.memory import estimate_training_memory

from . import dist_workers as W

pytestmark = pytest.mark.distributed

P = sum(p.numel() for p in MLP(W.MLP_CFG, seed=0).parameters())  # 1633


def _cfg(topology: dict, *, micro: int = 4, accumulation: int = 1, **extra: dict) -> dict:
    cfg = {"backend": "gloo", "device": "cpu", "topology": topology,
           "model": {"kind": "mlp", "input_size": 16, "hidden_size": 32, "num_layers": 2, "output_size": 1,
                     "activation": "relu"},
           "data": {"micro_batch_size": micro, "num_train_samples": 512, "num_eval_samples": 0},
           "optimizer": {"learning_rate": 1e-3},
           "training": {"max_steps": 3, "log_every_steps": 0, "gradient_accumulation_steps": accumulation}}
    cfg.update(extra)
    return cfg


def _run(world: int, cfg: dict) -> list[dict]:
    return [r.value for r in launch_workers(W.instrumented_engine_worker, world, args=(cfg, 3), timeout_seconds=300)]


def _op(comm: dict, prefix: str) -> tuple[int, int]:
    calls = sum(c for k, (c, _) in comm.items() if k.startswith(prefix))
    nbytes = sum(b for k, (_, b) in comm.items() if k.startswith(prefix))
    return calls, nbytes


@pytest.mark.parametrize("world", [2, 4])
def test_ddp_moves_each_gradient_once_per_step(world: int) -> None:
    v = _run(world, _cfg({"data_parallel_size": world}, ddp={"bucket_cap_mb": 0.002}))[0]
    calls, nbytes = _op(v["comm"], "all_reduce/data_parallel")
    assert nbytes == 4 * P  # every fp32 gradient exactly once
    assert calls >= 3  # one call per bucket (2 KB buckets)
    assert v["comm"]["all_reduce/dp_shard"] == (1, 4)  # and the step's loss, one fp32 scalar


def test_ddp_volume_is_independent_of_the_world_size() -> None:
    a = _op(_run(2, _cfg({"data_parallel_size": 2}))[0]["comm"], "all_reduce/data_parallel")[1]
    b = _op(_run(4, _cfg({"data_parallel_size": 4}))[0]["comm"], "all_reduce/data_parallel")[1]
    assert a == b == 4 * P


def test_bucket_size_changes_the_call_count_not_the_volume() -> None:
    seen = []
    for bucket_mb in (0.001, 0.004, 25.0):
        v = _run(2, _cfg({"data_parallel_size": 2}, ddp={"bucket_cap_mb": bucket_mb}))[0]
        calls, nbytes = _op(v["comm"], "all_reduce/data_parallel")
        assert nbytes == 4 * P, bucket_mb
        seen.append(calls)
    assert seen[0] > seen[1] > seen[2] == 1, seen  # a 25 MiB cap holds the whole model


def test_accumulation_keeps_one_reduction_per_step() -> None:
    one = _run(2, _cfg({"data_parallel_size": 2}, micro=4))[0]["comm"]
    two = _run(2, _cfg({"data_parallel_size": 2}, micro=2, accumulation=2))[0]["comm"]
    assert _op(one, "all_reduce/data_parallel") == _op(two, "all_reduce/data_parallel")


@pytest.mark.parametrize("reshard", [True, False])
def test_fsdp_gathers_per_pass_and_reduce_scatters_once(reshard: bool) -> None:
    world = 2
    v = _run(world, _cfg({"shard_parallel_size": world}, fsdp={"reshard_after_forward": reshard}))[0]
    ag_calls, ag_bytes = _op(v["comm"], "all_gather/shard")
    rs_calls, rs_bytes = _op(v["comm"], "reduce_scatter/shard")
    shard = -(-P // world)
    assert ag_calls == (2 if reshard else 1)  # forward (+ the refill in backward)
    assert ag_bytes == ag_calls * shard * 4
    assert rs_calls == 1 and rs_bytes == shard * world * 4


@pytest.mark.parametrize("world", [2, 4])
def test_fsdp_holds_a_shard_of_parameters_gradients_and_state(world: int) -> None:
    values = _run(world, _cfg({"shard_parallel_size": world}))
    shard = -(-P // world)
    for v in values:
        assert v["local_params"] == shard
        assert v["optimizer_elements"] == 2 * shard  # AdamW's two moments of the shard
        assert v["memory"]["grad_shard_bytes"] == 0  # gradients are released after the step
        assert v["memory"]["full_bytes"] == 0  # nothing stays gathered between steps
        est = estimate_training_memory(P, shard_group_size=world, largest_unit_parameters=v["largest_unit"])
        assert est.persistent_parameters == v["memory"]["shard_bytes"]
