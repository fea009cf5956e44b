"""Runtime tier on CPU/Gloo ranks: collective wrappers, context bring-up, launcher fault reporting,
PyTorch DDP as an oracle, tensor-parallel layers against full layers, hybrid sharding and the
communication volume of one step (bytes and call counts, never time).

Faults are injected on the host only: a rank that raises, and a rank that never reaches a
collective (the launcher's deadline names it).
"""

from __future__ import annotations

import pytest
import torch

from hybrid_training.distributed import WorkerFailure, launch_workers
from hybrid_training.distributed.context import LaunchEnvironment

from . import dist_workers as W
from . import runtime_workers as R

pytestmark = pytest.mark.distributed


@pytest.fixture(scope="module")
def collectives4() -> list:
    return launch_workers(R.collectives_worker, 4, timeout_seconds=300)


def test_all_reduce_ops(collectives4: list) -> None:
    ranks = [torch.arange(4, dtype=torch.float32) + 10 * r for r in range(4)]
    stacked = torch.stack(ranks)
    for r in collectives4:
        v = r.value
        assert torch.equal(v["all_reduce_sum"], stacked.sum(0))
        assert torch.allclose(v["all_reduce_avg"], stacked.mean(0), atol=1e-6)
        assert torch.equal(v["all_reduce_max"], stacked.max(0).values)
        assert torch.equal(v["all_reduce_min"], stacked.min(0).values)


def test_broadcast_gather_scatter_all_to_all(collectives4: list) -> None:
    world = 4
    full = sum(torch.arange(2 * world, dtype=torch.float32) + r for r in range(world))
    for r in collectives4:
        v = r.value
        tensor_group = [r.rank - r.rank % 2, r.rank - r.rank % 2 + 1]
        assert torch.equal(v["broadcast_from_local1"], torch.full((3,), float(tensor_group[1])))
        assert torch.equal(v["all_gather"], torch.tensor([[q, q] for q in range(world)], dtype=torch.float32))
        assert torch.equal(v["reduce_scatter_sum"], full[2 * r.rank:2 * r.rank + 2])
        assert torch.allclose(v["reduce_scatter_avg"], full[2 * r.rank:2 * r.rank + 2] / world, atol=1e-6)
        assert torch.equal(v["all_to_all"], torch.tensor([r.rank + 100 * q for q in range(world)], dtype=torch.float32))
        assert v["ring_received"] == float(tensor_group[(r.rank % 2 - 1) % 2])


def test_wrapper_errors_are_rank_aware(collectives4: list) -> None:
    for r in collectives4:
        v = r.value
        for key in ("reduce_scatter_indivisible", "send_to_self", "non_contiguous", "unknown_op", "bad_source"):
            assert v[key].startswith(f"[rank {r.rank}"), (key, v[key])
        assert "contiguous" in v["non_contiguous"] and "Fix:" in v["non_contiguous"]


def test_trivial_groups_short_circuit(collectives4: list) -> None:
    for r in collectives4:
        assert r.value["trivial_all_reduce_identity"] and r.value["trivial_all_gather_copy"]
        assert "all_reduce/sequence" not in r.value["recorder_keys"]


def test_recorder_counts_calls_bytes_and_waits(collectives4: list) -> None:
    for r in collectives4:
        v = r.value
        assert v["async_calls_delta"] == 1  # the wait does not count as a call
        assert {"all_reduce/world", "all_gather/world", "reduce_scatter/world", "all_to_all/world"} <= set(v["recorder_keys"])
        assert v["all_reduce_bytes"] == 5 * 4 * 4  # four ops + one async call of 4 fp32 values


def test_consistency_checks_raise_on_every_rank(collectives4: list) -> None:
    for r in collectives4:
        assert "layout differs across the 'world' group" in r.value["metadata_mismatch"]
        # data-parallel groups are (0, 2) and (1, 3); only rank 2 holds a value unlike its group's rank 0
        if r.rank == 2:
            assert "is not the same here as on the group's first rank" in r.value["tensor_mismatch"]
        else:
            assert r.value["tensor_mismatch"] == "NO ERROR"
        assert r.value["sum_scalar"] == 10.0
        assert [o["r"] for o in r.value["objects"]] == sorted(o["r"] for o in r.value["objects"])


def test_launcher_reports_the_failing_rank_with_its_traceback() -> None:
    with pytest.raises(WorkerFailure) as info:
        launch_workers(R.failing_worker, 2, args=("raise",), timeout_seconds=120)
    text = str(info.value)
    assert "failing ranks: [" in text and "1" in text
    results = launch_workers(R.failing_worker, 2, args=("raise",), timeout_seconds=120, raise_on_failure=False)
    assert not results[1].succeeded and "injected failure on rank 1" in (results[1].traceback_text or "")


def test_launcher_names_a_silent_rank_at_the_deadline() -> None:
    results = launch_workers(R.failing_worker, 2, args=("silent",), timeout_seconds=30, raise_on_failure=False)
    assert not results[1].succeeded
    assert "no result" in (results[1].traceback_text or "")


def test_context_refuses_double_init_and_builds_the_grid() -> None:
    results = launch_workers(R.context_worker, 4, timeout_seconds=300)
    for r in results:
        assert "already has an active distributed context" in r.value["again"]
    # rank = (dp * shard + sh) * 1 + 0 with shard innermost of the two
    assert results[3].value["shard"] == [2, 3] and results[3].value["data_parallel"] == [1, 3]
    assert results[3].value["dp_shard"] == [0, 1, 2, 3]


def test_bad_topology_fails_on_every_rank() -> None:
    results = launch_workers(R.bad_topology_worker, 2, timeout_seconds=120)
    for r in results:
        assert "TopologyError" in r.value or "ConfigurationError" in r.value, r.value


def test_launch_environment_parsing() -> None:
    env = {"RANK": "3", "WORLD_SIZE": "8", "LOCAL_RANK": "1", "LOCAL_WORLD_SIZE": "4", "MASTER_ADDR": "127.0.0.1",
           "MASTER_PORT": "29555"}
    launch = LaunchEnvironment.from_environment(env)
    assert (launch.rank, launch.world_size, launch.local_rank, launch.master_port) == (3, 8, 1, 29555)
    single = LaunchEnvironment.from_environment({}, allow_single_process=True)
    assert single.world_size == 1 and single.rank == 0
    with pytest.raises(Exception):
        LaunchEnvironment.from_environment({"RANK": "0"}, allow_single_process=False)


@pytest.mark.parametrize("world", [2, 4])
def test_ddp_matches_pytorch_ddp(world: int) -> None:
    results = launch_workers(R.torch_ddp_oracle_worker, world, args=(3,), timeout_seconds=300)
    for r in results:
        assert r.value["max_grad_diff"] <= 1e-7, r.value
        assert r.value["layouts"] > 1


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_layers_match_full_layers(world: int) -> None:
    results = launch_workers(R.tp_layers_worker, world, timeout_seconds=300)
    for r in results:
        v = r.value
        assert v["column_full_weight"] == 0.0 and v["row_full_weight"] == 0.0
        assert v["column_forward"] == 0.0 and v["column_weight_grad"] < 1e-5
        assert v["column_input_grad"] < 1e-5 and v["row_forward"] < 1e-5
        assert v["embedding_forward"] == 0.0


def test_hybrid_sharding_matches_single_process() -> None:
    steps = 3
    ref = W.single_process_mlp(4, steps=steps)  # four data ranks: dp_shard spans dp x shard
    results = launch_workers(R.hsdp_worker, 4, args=(steps,), timeout_seconds=300)
    for r in results:
        assert {"reduce_scatter/shard", "all_reduce/data_parallel", "all_gather/shard"} <= set(r.value["ops"])
        for name, p in ref["params"].items():
            assert torch.allclose(r.value["full"][name], p, atol=1e-5), name


def test_communication_volume_per_step() -> None:
    """DDP moves the gradients once (4P bytes fp32); FSDP gathers twice and reduce-scatters once with reshard."""
    ddp = launch_workers(R.comm_volume_worker, 2, args=("ddp", True), timeout_seconds=300)[0].value
    assert ddp["ops"]["all_reduce/data_parallel"][1] == 4 * ddp["params"]
    fsdp = launch_workers(R.comm_volume_worker, 2, args=("fsdp", True), timeout_seconds=300)[0].value
    shard_bytes = fsdp["padded"] // 2 * 4
    assert fsdp["ops"]["all_gather/shard"] == (2, 2 * shard_bytes)  # forward gather + backward refill
    assert fsdp["ops"]["reduce_scatter/shard"][0] == 1
    keep = launch_workers(R.comm_volume_worker, 2, args=("fsdp", False), timeout_seconds=300)[0].value
    assert keep["ops"]["all_gather/shard"][0] == 1  # no refill without reshard_after_forward


def test_launcher_exports_the_rendezvous_environment() -> None:
    results = launch_workers(R.env_probe_worker, 2, timeout_seconds=120)
    assert [r.value["RANK"] for r in results] == ["0", "1"]
    assert all(r.value["WORLD_SIZE"] == "2" and r.value["MASTER_ADDR"] == "127.0.0.1" for r in results)


@pytest.mark.parametrize("kind,algorithm,world", [("gpt2", "all_gather", 2), ("llama", "all_gather", 2), ("gpt2", "ring", 2),
                                                  ("llama", "ring", 4), ("gpt2", "ulysses", 2), ("llama", "ulysses", 2),
                                                  ("gpt2", "ulysses", 4)])
def test_independent_sequence_parallel_matches_single_process(kind: str, algorithm: str, world: int) -> None:
    """``independent`` mode is context parallelism: every chunk attends to the whole prefix (all-gather, ring or Ulysses)."""
    ref = launch_workers(W.transformer_forward_worker, 1, args=(1, False, kind), timeout_seconds=300)[0].value
    for r in launch_workers(R.independent_sp_worker, world, args=(kind, algorithm), timeout_seconds=300):
        assert abs(r.value["loss"] - ref["loss"]) < 1e-5
        assert torch.allclose(r.value["logits"], ref["logits"], atol=1e-5)
        assert set(r.value["grads"]) == set(ref["grads"])
        for name, g in ref["grads"].items():
            assert torch.allclose(r.value["grads"][name], g, atol=1e-5), name


def test_engine_with_context_parallel_trains_like_data_parallel_alone(tmp_path) -> None:
    """dp2 x seq2 (independent) sees the same global batch as dp2; their losses and weights agree."""
    base = {"backend": "gloo", "device": "cpu",
            "model": {"kind": "transformer", "hidden_size": 32, "num_layers": 2, "num_heads": 4, "vocab_size": 64,
                      "max_sequence_length": 16},
            "data": {"micro_batch_size": 2, "sequence_length": 16, "num_train_samples": 64, "num_eval_samples": 0,
                     "shuffle": False},
            "optimizer": {"learning_rate": 0.003}, "training": {"max_steps": 3, "log_every_steps": 0}}
    dp = dict(base, topology={"data_parallel_size": 2})
    cp = dict(base, topology={"data_parallel_size": 2, "sequence_parallel_size": 2, "sequence_parallel_mode": "independent"},
              tensor_parallel={"sequence_parallel": True})
    ref = launch_workers(W.engine_worker, 2, args=(dp, 3, None, None), timeout_seconds=300)[0].value
    got = launch_workers(W.engine_worker, 4, args=(cp, 3, None, None), timeout_seconds=300)
    for r in got:
        for a, b in zip(r.value["losses"], ref["losses"]):
            assert abs(a - b) < 1e-5, (r.value["losses"], ref["losses"])
        diffs = {}
        for name, t in ref["full"].items():
            mine = r.value["full"][name]
            if name.endswith("qkv.bias"):
                # The key bias shifts every score of a query row equally, so softmax makes its gradient
                # exactly zero; the computed values are rounding noise that AdamW normalises to steps of
                # the learning rate's size in either direction.  Compare the query and value biases.
                mine, t = torch.cat([mine[:32], mine[64:]]), torch.cat([t[:32], t[64:]])
            diffs[name] = float((mine - t).abs().max())
        assert max(diffs.values()) < 1e-5, sorted(diffs.items(), key=lambda kv: -kv[1])[:4]
