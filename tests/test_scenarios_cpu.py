"""End-to-end scenarios through the real engine on CPU/Gloo ranks, each with a numerical assertion.

The scenarios of the reference suite (``tests/end_to_end/test_training_scenarios.py``): the
single-process baseline, DDP and FSDP at two ranks, tensor and sequence parallelism of the
transformer at two ranks, the four-rank hybrid grid; checkpoint resume and resharding are in
``test_checkpoint.py``.  The global batch is held constant across world sizes, so every run
consumes the same samples and the final weights are comparable.
"""

from __future__ import annotations

import pytest
import torch

from hybrid_training.distributed import launch_workers

from . import dist_workers as W

pytestmark = pytest.mark.distributed

GLOBAL_BATCH = 8
STEPS = 6
TOL = 1e-5  # after optimizer steps, different reduction orders


def _mlp(topology: dict, replicas: int, **extra: dict) -> dict:
    cfg = {"backend": "gloo", "device": "cpu", "topology": topology,
           "model": {"kind": "mlp", "input_size": 12, "hidden_size": 20, "num_layers": 3, "output_size": 6},
           "data": {"micro_batch_size": GLOBAL_BATCH // replicas, "num_train_samples": 256, "num_eval_samples": 0,
                    "shuffle": False},
           "optimizer": {"learning_rate": 3e-3}, "training": {"max_steps": STEPS, "log_every_steps": 0}}
    cfg.update(extra)
    return cfg


def _transformer(topology: dict, replicas: int, **extra: dict) -> dict:
    cfg = {"backend": "gloo", "device": "cpu", "topology": topology,
           "model": {"kind": "transformer", "vocab_size": 32, "hidden_size": 16, "num_heads": 4, "num_layers": 2,
                     "ffn_hidden_size": 32, "max_sequence_length": 16},
           "data": {"micro_batch_size": GLOBAL_BATCH // replicas, "sequence_length": 16, "num_train_samples": 256,
                    "num_eval_samples": 0, "shuffle": False},
           "optimizer": {"learning_rate": 3e-3}, "training": {"max_steps": STEPS, "log_every_steps": 0}}
    cfg.update(extra)
    return cfg


def _train(world: int, cfg: dict) -> list[dict]:
    return [r.value for r in launch_workers(W.engine_worker, world, args=(cfg, STEPS, None, None), timeout_seconds=600)]


@pytest.fixture(scope="module")
def mlp_baseline() -> dict:
    return _train(1, _mlp({}, 1))[0]


@pytest.fixture(scope="module")
def transformer_baseline() -> dict:
    return _train(1, _transformer({}, 1))[0]


def _assert_same(run: dict, base: dict, tol: float = TOL) -> None:
    for name, t in base["full"].items():
        got = run["full"][name]
        if name.endswith("qkv.bias"):
            # The key bias adds the same amount to every score of a query row, which the softmax
            # cancels: its gradient is rounding noise, which Adam scales up to learning-rate-sized
            # steps, so only the query and value thirds are comparable.
            third = t.numel() // 3
            keep = torch.cat([torch.arange(third), torch.arange(2 * third, 3 * third)])
            got, t = got[keep], t[keep]
        assert torch.allclose(got, t, atol=tol), (name, float((got - t).abs().max()))
    for a, b in zip(run["losses"], base["losses"]):
        assert abs(a - b) < 1e-4 * max(1.0, abs(b)), (run["losses"], base["losses"])


def test_single_process_baseline_learns(mlp_baseline: dict) -> None:
    losses = mlp_baseline["losses"]
    assert len(losses) == STEPS and all(l == l for l in losses)
    assert losses[-1] < losses[0], losses


@pytest.mark.parametrize(("strategy", "topology"), [("ddp", {"data_parallel_size": 2}),
                                                    ("fsdp", {"shard_parallel_size": 2})])
def test_two_rank_data_parallel_strategies_match_the_baseline(strategy: str, topology: dict, mlp_baseline: dict) -> None:
    runs = _train(2, _mlp(topology, 2))
    for r in runs:
        _assert_same(r, mlp_baseline)
    assert runs[0]["losses"] == runs[1]["losses"], "both ranks report the same reduced loss"


def test_four_rank_hybrid_grid_matches_the_baseline(mlp_baseline: dict) -> None:
    runs = _train(4, _mlp({"data_parallel_size": 2, "shard_parallel_size": 2}, 4))
    for r in runs:
        _assert_same(r, mlp_baseline)


@pytest.mark.parametrize(("strategy", "topology", "tp"), [
    ("tensor", {"tensor_parallel_size": 2}, {}),
    ("tensor+sequence", {"tensor_parallel_size": 2, "sequence_parallel_mode": "tensor_group"}, {"sequence_parallel": True}),
])
def test_two_rank_model_parallel_transformer_matches_the_baseline(strategy: str, topology: dict, tp: dict,
                                                                  transformer_baseline: dict) -> None:
    runs = _train(2, _transformer(topology, 1, tensor_parallel=tp))
    for r in runs:
        _assert_same(r, transformer_baseline, tol=1e-4)  # TP reorders sums; Adam amplifies tiny gradients
    assert transformer_baseline["losses"][-1] < transformer_baseline["losses"][0]


def test_data_parallel_plus_tensor_parallel_transformer_matches_the_baseline(transformer_baseline: dict) -> None:
    runs = _train(4, _transformer({"data_parallel_size": 2, "tensor_parallel_size": 2, "sequence_parallel_mode": "tensor_group"},
                                  2, tensor_parallel={"sequence_parallel": True}))
    for r in runs:
        _assert_same(r, transformer_baseline, tol=1e-4)
