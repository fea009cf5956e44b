"""Multi-process numerical equivalence on CPU/Gloo ranks (the oracle tier).

Every distributed strategy is compared against a single-process run that sees
the same global batch with the same seeds: DDP, no_sync accumulation, unused
parameter handling, FSDP (the 1633-parameter MLP of the benchmark config:
shard 409, padding 3 at world 4), tensor parallelism and sequence parallelism
of the transformer (GPT-2 and Llama variants), and the engine end to end.
"""

from __future__ import annotations

import pytest
import torch

from hybrid_training.distributed import launch_workers

from . import dist_workers as W

pytestmark = pytest.mark.distributed


@pytest.mark.parametrize("world", [2, 4])
def test_ddp_matches_single_process(world: int) -> None:
    ref = W.single_process_mlp(world, steps=3)
    results = launch_workers(W.ddp_mlp_worker, world, args=(3, 0.001), timeout_seconds=300)
    for r in results:
        for name, g in r.value["grads0"].items():
            assert torch.allclose(g, ref["grads0"][name], atol=1e-6), name
        for name, p in r.value["params"].items():
            assert torch.allclose(p, ref["params"][name], atol=1e-5), name
    assert results[0].value["buckets"] > 1
    assert results[0].value["stats"]["buckets_reduced"] == 3 * results[0].value["buckets"]


def test_ddp_no_sync_accumulation_equals_large_batch() -> None:
    world = 2
    results = launch_workers(W.ddp_no_sync_worker, world, timeout_seconds=300)
    from hybrid_training.models import MLP

    model = MLP(W.MLP_CFG, seed=0)
    xs, ys = zip(*(W.mlp_batch(0, r, per_rank=8) for r in range(world)))
    torch.nn.functional.mse_loss(model(torch.cat(xs)), torch.cat(ys)).backward()
    for name, p in model.named_parameters():
        assert torch.allclose(results[0].value[name], p.grad, atol=1e-6), name


def test_ddp_unused_parameters() -> None:
    bad = launch_workers(W.ddp_unused_worker, 2, args=(False,), timeout_seconds=300)
    assert all(r.value == "error:ShardingError" for r in bad)
    ok = launch_workers(W.ddp_unused_worker, 2, args=(True,), timeout_seconds=300)
    assert all(r.value.startswith("ok:") and "unused" in r.value for r in ok)


@pytest.mark.parametrize("world,shard,pad", [(2, 817, 1), (4, 409, 3)])
def test_fsdp_matches_single_process(world: int, shard: int, pad: int) -> None:
    steps = 5
    ref = W.single_process_mlp(world, steps=steps)
    results = launch_workers(W.fsdp_mlp_worker, world, args=(steps,), timeout_seconds=300)
    for r in results:
        assert r.value["shard"] == shard and r.value["padding"] == pad and r.value["full_bytes"] == 0
        for name, p in ref["params"].items():
            assert torch.allclose(r.value["full"][name], p, atol=1e-5), name


@pytest.mark.parametrize("kind", ["gpt2", "llama"])
@pytest.mark.parametrize("tp,sp", [(2, False), (2, True)])
def test_tensor_and_sequence_parallel_match_single_process(kind: str, tp: int, sp: bool) -> None:
    ref = launch_workers(W.transformer_forward_worker, 1, args=(1, False, kind), timeout_seconds=300)[0].value
    results = launch_workers(W.transformer_forward_worker, tp, args=(tp, sp, kind), timeout_seconds=300)
    for r in results:
        assert abs(r.value["loss"] - ref["loss"]) < 1e-5
        assert torch.allclose(r.value["logits"], ref["logits"], atol=1e-5)
        for name, g in ref["grads"].items():
            assert torch.allclose(r.value["grads"][name], g, atol=1e-5), name


def _engine_cfg(topology: dict, **extra: dict) -> dict:
    cfg = {"backend": "gloo", "device": "cpu", "topology": topology,
           "model": {"kind": "transformer", "hidden_size": 32, "num_layers": 2, "num_heads": 4, "vocab_size": 64,
                     "max_sequence_length": 16},
           "data": {"micro_batch_size": 2, "sequence_length": 16, "num_train_samples": 256, "num_eval_samples": 0},
           "optimizer": {"learning_rate": 0.003}, "training": {"max_steps": 4, "log_every_steps": 0, "max_grad_norm": 1.0}}
    cfg.update(extra)
    return cfg


def test_engine_hybrid_grid_trains(tmp_path) -> None:
    topo = {"data_parallel_size": 2, "shard_parallel_size": 2, "tensor_parallel_size": 2, "sequence_parallel_mode": "tensor_group"}
    cfg = _engine_cfg(topo, tensor_parallel={"sequence_parallel": True}, fsdp={"auto_wrap_min_num_params": 1000})
    results = launch_workers(W.engine_worker, 8, args=(cfg, 4, None, None), timeout_seconds=600)
    losses = [r.value["losses"] for r in results]
    assert all(l == losses[0] for l in losses), "every rank must report the same reduced loss"
    assert all(torch.isfinite(torch.tensor(l)).all() for l in losses)
