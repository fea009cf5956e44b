"""The training engine on one B200: the optimizer update overlapped with the backward pass.

With no clipping, no gradient-norm metric and no loss scaling, the engine applies AdamW to each
group of parameters as soon as the backward pass has written their gradients (on a side stream,
with the small-footprint update kernel).  The result must match the step that runs AdamW once
after the backward pass, eagerly and when the step is replayed from a CUDA graph.
"""

from __future__ import annotations

import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _train(overlap: bool, graph: bool, steps: int = 4) -> tuple[list[float], dict[str, torch.Tensor]]:
    from hybrid_training.config import ExperimentConfig
    from hybrid_training.distributed.context import init_distributed
    from hybrid_training.training.engine import TrainingEngine

    cfg = ExperimentConfig.from_dict({
        "name": "overlap-test", "backend": "nccl", "device": "cuda", "timeout_seconds": 120.0,
        "model": {"kind": "transformer", "hidden_size": 128, "num_layers": 2, "num_heads": 2, "vocab_size": 512,
                  "max_sequence_length": 64, "tie_word_embeddings": True},
        "data": {"micro_batch_size": 4, "sequence_length": 64, "num_train_samples": 4096, "num_eval_samples": 0,
                 "shuffle": False},
        "optimizer": {"learning_rate": 1e-3},
        "mixed_precision": {"enabled": True, "param_dtype": "bfloat16"},
        "ddp": {"bucket_cap_mb": 0.05},
        "training": {"max_steps": steps, "log_every_steps": 0, "overlap_optimizer_step": overlap, "cuda_graph": graph}})
    ctx = init_distributed(cfg)
    try:
        engine = TrainingEngine(cfg, ctx)
        assert (engine.overlapped_step is not None) == overlap
        engine.train(max_steps=steps)
        params = {n: p.detach().float().cpu().clone() for n, p in engine.model.named_parameters()}
        losses = [m.loss for m in engine.history]
        engine.close()
        return losses, params
    finally:
        ctx.shutdown()


@pytest.mark.parametrize("graph", [False, True])
def test_overlapped_update_matches_the_update_after_the_backward(graph: bool, monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setenv("MASTER_ADDR", "127.0.0.1")
    base_losses, base = _train(False, graph)
    losses, params = _train(True, graph)
    for name, ref in base.items():
        assert torch.allclose(params[name], ref, atol=2e-3, rtol=2e-3), (name, float((params[name] - ref).abs().max()))
    for a, b in zip(losses, base_losses):
        assert abs(a - b) < 1e-2 * max(1.0, abs(b)), (losses, base_losses)
    assert all(x == x for x in losses)


def test_resident_adamw_kernel_matches_the_regular_one() -> None:
    import hybrid_training.ops as ops

    dev = torch.device("cuda")
    n = 1_000_064
    gen = torch.Generator(device=dev).manual_seed(3)
    p0 = torch.randn(n, device=dev, generator=gen)
    g = torch.randn(n, device=dev, generator=gen)
    m0 = torch.randn(n, device=dev, generator=gen) * 0.1
    v0 = torch.rand(n, device=dev, generator=gen) * 0.1
    hyper = torch.tensor([1e-2, 3.0, 0.5, 0.0], device=dev)
    outs = []
    for resident in (False, True):
        p, m, v = p0.clone(), m0.clone(), v0.clone()
        copy = torch.empty(n, device=dev, dtype=torch.bfloat16)
        ops.adamw_flat(p, g, m, v, copy, hyper, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, resident=resident)
        outs.append((p, m, v, copy))
    for a, b in zip(*outs):
        assert torch.equal(a, b)  # the same arithmetic per element
    # A 64-element-aligned slice in the middle, as the overlapped step updates it.
    p, m, v = p0.clone(), m0.clone(), v0.clone()
    ops.adamw_flat(p[640:6400], g[640:6400], m[640:6400], v[640:6400], None, hyper, beta1=0.9, beta2=0.95, eps=1e-8,
                   weight_decay=0.1, resident=True)
    assert torch.equal(p[640:6400], outs[0][0][640:6400]) and torch.equal(p[:640], p0[:640]) and torch.equal(p[6400:], p0[6400:])
