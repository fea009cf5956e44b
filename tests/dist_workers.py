"""Module-level worker functions for multi-process (Gloo/CPU) tests.

Each worker runs inside a rank spawned by ``launch_workers`` and returns
plain Python / CPU tensors for the parent to compare against a single-process
reference computed with the same seeds.
"""

from __future__ import annotations

import os

import dataclasses
from pathlib import Path
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from hybrid_training.config import (
    CheckpointConfig,
    DataConfig,
    DDPConfig,
    ExperimentConfig,
    FSDPConfig,
    ModelConfig,
    OptimizerConfig,
    TopologyConfig,
    TrainingConfig,
)
from hybrid_training.distributed import CommunicationRecorder, init_distributed
from hybrid_training.models import MLP
from hybrid_training.parallel import DistributedDataParallel, FullyShardedDataParallel
from hybrid_training.training import TrainingEngine

MLP_CFG = ModelConfig(kind="mlp", input_size=16, hidden_size=32, num_layers=2, output_size=1, activation="relu")


def mlp_batch(step: int, rank: int, per_rank: int = 8) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator().manual_seed(1000 * step + rank)
    return torch.randn(per_rank, 16, generator=g), torch.randn(per_rank, 1, generator=g)


def single_process_mlp(world: int, steps: int, lr: float = 1e-3) -> dict[str, Any]:
    """The reference run: one process sees the concatenation of every rank's batch."""
    model = MLP(MLP_CFG, seed=0)
    opt = torch.optim.AdamW(model.parameters(), lr=lr, weight_decay=0.0)
    grads = None
    for step in range(steps):
        xs, ys = zip(*(mlp_batch(step, r) for r in range(world)))
        x, y = torch.cat(xs), torch.cat(ys)
        opt.zero_grad()
        F.mse_loss(model(x), y).backward()
        if step == 0:
            grads = {n: p.grad.clone() for n, p in model.named_parameters()}
        opt.step()
    return {"params": {n: p.detach().clone() for n, p in model.named_parameters()}, "grads0": grads}


def ddp_mlp_worker(rank: int, world: int, steps: int, bucket_mb: float) -> dict[str, Any]:
    ctx = init_distributed(TopologyConfig(data_parallel_size=world), backend="gloo", device="cpu")
    try:
        model = MLP(MLP_CFG, seed=0)
        recorder = CommunicationRecorder()
        ddp = DistributedDataParallel(model, ctx.group("data_parallel"), DDPConfig(bucket_cap_mb=bucket_mb), recorder=recorder)
        from hybrid_training.optim import FusedAdamW

        opt = FusedAdamW(ddp.parameters(), lr=1e-3, weight_decay=0.0)
        grads0 = None
        for step in range(steps):
            x, y = mlp_batch(step, rank)
            F.mse_loss(ddp(x), y).backward()
            ddp.finish_gradient_synchronization()
            if step == 0:
                grads0 = {n: p.grad.clone() for n, p in model.named_parameters()}
            opt.step()
            opt.zero_grad()
        return {"params": {n: p.detach().clone() for n, p in model.named_parameters()}, "grads0": grads0,
                "buckets": len(ddp.bucket_layouts()), "calls": recorder.total().calls,
                "stats": ddp.statistics.as_dict()}
    finally:
        ctx.shutdown()


def ddp_no_sync_worker(rank: int, world: int) -> dict[str, Any]:
    """Two accumulated micro-batches under no_sync equal one batch of twice the size."""
    ctx = init_distributed(TopologyConfig(data_parallel_size=world), backend="gloo", device="cpu")
    try:
        model = MLP(MLP_CFG, seed=0)
        ddp = DistributedDataParallel(model, ctx.group("data_parallel"), DDPConfig(bucket_cap_mb=0.01))
        x, y = mlp_batch(0, rank, per_rank=8)
        with ddp.no_sync():
            (F.mse_loss(ddp(x[:4]), y[:4]) / 2).backward()
        (F.mse_loss(ddp(x[4:]), y[4:]) / 2).backward()
        ddp.finish_gradient_synchronization()
        return {n: p.grad.clone() for n, p in model.named_parameters()}
    finally:
        ctx.shutdown()


def ddp_unused_worker(rank: int, world: int, find_unused: bool) -> str:
    ctx = init_distributed(TopologyConfig(data_parallel_size=world), backend="gloo", device="cpu")
    try:
        model = nn.ModuleDict({"used": nn.Linear(4, 4), "unused": nn.Linear(4, 4)})

        class Wrapper(nn.Module):
            def __init__(self) -> None:
                super().__init__()
                self.m = model

            def forward(self, x: torch.Tensor) -> torch.Tensor:
                return self.m["used"](x)

        ddp = DistributedDataParallel(Wrapper(), ctx.group("data_parallel"), DDPConfig(find_unused_parameters=find_unused))
        ddp(torch.randn(2, 4)).sum().backward()
        try:
            ddp.finish_gradient_synchronization()
        except Exception as exc:  # noqa: BLE001
            return f"error:{type(exc).__name__}"
        return "ok:" + ",".join(ddp.statistics.unused_parameters)
    finally:
        ctx.shutdown()


def fsdp_mlp_worker(rank: int, world: int, steps: int) -> dict[str, Any]:
    ctx = init_distributed(TopologyConfig(shard_parallel_size=world), backend="gloo", device="cpu")
    try:
        model = MLP(MLP_CFG, seed=0)
        fsdp = FullyShardedDataParallel(model, ctx.group("shard"))
        from hybrid_training.optim import FusedAdamW

        opt = FusedAdamW([fsdp.handle.flat_param], lr=1e-3, weight_decay=0.0)
        for step in range(steps):
            x, y = mlp_batch(step, rank)
            F.mse_loss(fsdp(x), y).backward()
            fsdp.finish_backward()
            opt.step()
            opt.zero_grad()
        full = fsdp.full_state_dict()
        return {"full": full, "shard": fsdp.handle.shard_numel, "padding": fsdp.handle.padding,
                "full_bytes": fsdp.memory_summary()["full_bytes"]}
    finally:
        ctx.shutdown()


def _tiny_transformer(kind: str = "gpt2") -> ModelConfig:
    if kind == "llama":
        return ModelConfig.llama_1b3(hidden_size=32, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_size=48,
                                     vocab_size=64, max_sequence_length=16)
    return ModelConfig(kind="transformer", hidden_size=32, num_layers=2, num_heads=4, vocab_size=64, max_sequence_length=16)


def transformer_forward_worker(rank: int, world: int, tp: int, sp: bool, kind: str) -> dict[str, Any]:
    """Loss, logits and a few gradients of the transformer at TP width ``tp`` (optionally with SP)."""
    topo = TopologyConfig(tensor_parallel_size=tp, data_parallel_size=world // tp,
                          sequence_parallel_mode="tensor_group" if sp else "disabled")
    cfg = ExperimentConfig(backend="gloo", device="cpu", topology=topo, model=_tiny_transformer(kind),
                           tensor_parallel=dataclasses.replace(ExperimentConfig().tensor_parallel, sequence_parallel=sp))
    ctx = init_distributed(cfg)
    try:
        from hybrid_training.parallel import build_model

        model = build_model(cfg, ctx)
        g = torch.Generator().manual_seed(7)
        tokens = torch.randint(0, 64, (2, 17), generator=g)
        logits = model(tokens[:, :-1])
        loss = model(tokens[:, :-1], targets=tokens[:, 1:])
        loss.backward()
        if sp:
            from hybrid_training.parallel import all_reduce_sequence_parallel_gradients

            all_reduce_sequence_parallel_gradients(model, ctx.group("tensor"))
        grads = {}
        for name, p in model.named_parameters():
            if p.grad is not None and ("input_norm.weight" in name or "qkv.weight" in name):
                full = p.grad
                if getattr(p, "tensor_parallel_partition_dim", None) is not None and tp > 1:
                    from hybrid_training.autograd import all_gather_along_dim

                    full = all_gather_along_dim(p.grad.contiguous(), ctx.group("tensor"), p.tensor_parallel_partition_dim)
                    if "qkv" in name:
                        owner = model.get_submodule(name.rsplit(".", 1)[0])
                        full = owner.canonical(full)
                grads[name] = full.clone()
        return {"loss": float(loss.detach()), "logits": logits.detach().clone(), "grads": grads}
    finally:
        ctx.shutdown()


def _tensor_parallel_full(engine: Any, ctx: Any) -> dict[str, torch.Tensor]:
    """The model's full state with tensor-parallel slices gathered back into whole tensors."""
    full = engine.model.full_state_dict()
    tensor = ctx.group("tensor")
    if tensor.size == 1:
        return full
    from hybrid_training.autograd import all_gather_along_dim

    info = engine.model.parameter_parallel_info()
    inner = getattr(engine.model, "_inner_model", engine.model)
    out = {}
    for name, t in full.items():
        i = info.get(name)
        if i is not None and i.partition_dim is not None and i.tensor_parallel_size > 1:
            t = all_gather_along_dim(t.contiguous(), tensor, i.partition_dim)
            try:
                owner = inner.get_submodule(name.rsplit(".", 1)[0])
            except AttributeError:
                owner = None
            if owner is not None and hasattr(owner, "canonical"):
                t = owner.canonical(t)
        out[name] = t
    return out


def engine_worker(rank: int, world: int, overrides: dict[str, Any], steps: int, ckpt: str | None, resume: str | None) -> dict[str, Any]:
    cfg = ExperimentConfig.from_dict(overrides)
    ctx = init_distributed(cfg)
    try:
        engine = TrainingEngine(cfg, ctx)
        if resume:
            engine.load_checkpoint(resume)
        engine.train(max_steps=steps)
        path = str(engine.save_checkpoint(ckpt)) if ckpt else None
        full = _tensor_parallel_full(engine, ctx)
        out = {"losses": [m.loss for m in engine.history], "path": path,
               "full": {k: v.detach().clone() for k, v in full.items()}, "step": engine.state.step}
        engine.close()
        return out
    finally:
        ctx.shutdown()


def _cuda_experiment(world: int, *, fused: bool = True, steps: int = 3, overlap: bool = False,
                     graph: bool = False) -> dict[str, Any]:
    return {"name": "multigpu-test", "backend": "nccl", "device": "cuda", "timeout_seconds": 120.0,
            "topology": {"data_parallel_size": world},
            "model": {"kind": "transformer", "hidden_size": 128, "num_layers": 2, "num_heads": 2, "vocab_size": 512,
                      "max_sequence_length": 64},
            "data": {"micro_batch_size": 4, "sequence_length": 64, "num_train_samples": 4096, "num_eval_samples": 0,
                     "shuffle": False},
            "optimizer": {"learning_rate": 1e-3},
            "mixed_precision": {"enabled": True, "param_dtype": "bfloat16"},
            "ddp": {"bucket_cap_mb": 0.05, "fused_allreduce": fused},
            "training": {"max_steps": steps, "log_every_steps": 0, "overlap_optimizer_step": overlap, "cuda_graph": graph}}


def gathered_attention_worker(rank: int, world: int) -> dict[str, float]:
    """Native all-gather context-parallel attention of one chunk per rank against the single-GPU kernel
    over the whole sequence (output, and the gradient of this rank's chunk of the packed input)."""
    from hybrid_training import ops
    from hybrid_training.parallel.context_parallel import gathered_attention

    cfg = ExperimentConfig.from_dict(_cuda_experiment(world))
    ctx = init_distributed(cfg)
    try:
        torch.manual_seed(0)
        b, s, h, hkv, d = 2, 512 * world, 8, 4, 64
        qkv = (torch.randn(b, s, (h + 2 * hkv) * d, device=ctx.device) * 0.5).bfloat16()
        dout = torch.randn(b, s, h * d, device=ctx.device).bfloat16()
        local = s // world
        win = slice(rank * local, (rank + 1) * local)
        mine = qkv[:, win].clone().requires_grad_(True)
        out = gathered_attention(mine, h, hkv, d, ctx.group("data_parallel"), causal=True)
        out.backward(dout[:, win])
        full = qkv.clone().requires_grad_(True)
        ref = ops.attention(full, h, hkv, d, causal=True)
        ref.backward(dout)

        def rel(a: torch.Tensor, r: torch.Tensor) -> float:
            return float((a.float() - r.float()).norm() / r.float().norm())

        return {"out": rel(out, ref[:, win]), "dq": rel(mine.grad[..., : h * d], full.grad[:, win, : h * d]),
                "dkv": rel(mine.grad[..., h * d:], full.grad[:, win, h * d:])}
    finally:
        ctx.shutdown()


def bucket_allreduce_worker(rank: int, world: int, nvls: bool = False) -> dict[str, Any]:
    """In-kernel bucket all-reduce over NVLink peer memory against NCCL's all-reduce (average).

    ``nvls=True`` selects the NVLink-switch path (``multimem.ld_reduce`` / ``multimem.st``); the
    result then records whether the switch offered a multicast address at all.
    """
    import torch.distributed as dist

    from hybrid_training.ops.comm import bucket_all_reduce, nvls_available

    cfg = ExperimentConfig.from_dict(_cuda_experiment(world))
    ctx = init_distributed(cfg)
    try:
        ws = ctx.symmetric_workspace("data_parallel")
        assert ws is not None, "symmetric memory is unavailable"
        if nvls:
            os.environ["HT_NVLS"] = "1"
        numel = 3_000_011
        flat = ws.allocate(numel + 5, torch.float32)
        gen = torch.Generator(device="cuda").manual_seed(100 + rank)
        errors = []
        cases = zip(((0, numel), (4, 1001), (1024, 17), (8, 2_000_000), (0, numel), (8, 999_999), (0, numel), (12, 777_777)),
                    (True, True, False, False, False, True, False, True), (0, 0, 0, 0, 0, 0, 8, 8))
        for (start, n), wide, slots in cases:  # slots 8: the 8-peer instantiation run by two ranks
            flat.normal_(generator=gen)
            expect = flat[start:start + n].clone()
            dist.all_reduce(expect, op=dist.ReduceOp.SUM, group=ctx.group("data_parallel").process_group)
            expect /= world
            outside = torch.cat([flat[:start], flat[start + n:]]).clone()
            bucket_all_reduce(ws, flat, start, n, 1.0 / world, wide=wide, peer_slots=slots)
            torch.cuda.synchronize()
            ws.check_status()
            errors.append(float((flat[start:start + n] - expect).abs().max()))
            assert torch.equal(torch.cat([flat[:start], flat[start + n:]]), outside), "wrote outside the bucket"
        return {"errors": errors, "nvls": nvls and nvls_available(ws, flat)}
    finally:
        ctx.shutdown()


def ddp_cuda_worker(rank: int, world: int, fused: bool, steps: int, overlap: bool = False,
                    graph: bool = False) -> dict[str, Any]:
    """A few DDP steps on CUDA; returns the losses and the final parameters.

    ``overlap`` applies AdamW per bucket during the backward pass; ``graph`` replays the step
    from a CUDA graph after the warm-up steps.
    """
    cfg = ExperimentConfig.from_dict(_cuda_experiment(world, fused=fused, steps=steps, overlap=overlap, graph=graph))
    ctx = init_distributed(cfg)
    try:
        engine = TrainingEngine(cfg, ctx)
        ddp = getattr(engine.model, "_ddp", None)
        used_fused = ddp is not None and getattr(ddp, "_workspace", None) is not None
        assert (engine.overlapped_step is not None) == overlap
        engine.train(max_steps=steps)
        full = engine.model.full_state_dict()
        out = {"losses": [m.loss for m in engine.history], "fused": used_fused,
               "full": {k: v.detach().float().cpu().clone() for k, v in full.items()}}
        engine.close()
        return out
    finally:
        ctx.shutdown()


def tp_fused_collectives_worker(rank: int, world: int, sp: bool = True) -> dict[str, Any]:
    """Column- and row-parallel linears with the fused collective kernels against the NCCL path:
    with sequence parallelism (all-gather GEMM, GEMM reduce-scatter) or without it (in-kernel
    all-reduces of the row output and of the column input gradient)."""
    from hybrid_training.parallel.tensor_parallel import ColumnParallelLinear, RowParallelLinear

    cfg = ExperimentConfig.from_dict({
        "name": "tp-fused", "backend": "nccl", "device": "cuda", "timeout_seconds": 120.0,
        "topology": {"tensor_parallel_size": world, "sequence_parallel_mode": "tensor_group" if sp else "disabled"},
        "tensor_parallel": {"sequence_parallel": sp, "fused_collectives": True},
        "mixed_precision": {"enabled": True, "param_dtype": "bfloat16"},
        "model": {"kind": "transformer", "hidden_size": 256, "num_layers": 1, "num_heads": 4, "vocab_size": 512,
                  "max_sequence_length": 128 * world}})
    ctx = init_distributed(cfg)
    try:
        group = ctx.group("tensor")
        dev = ctx.device
        b, r, k, n = 2, 128, 256, 512
        col = ColumnParallelLinear(k, n, group, bias=True, sequence_parallel=sp, activation="gelu", init_seed=3, device=dev)
        row = RowParallelLinear(n, k, group, bias=True, sequence_parallel=sp, init_seed=4, device=dev)
        gen = torch.Generator(device="cpu").manual_seed(7)
        x_full = torch.randn(b, r * world, k, generator=gen)
        g_full = torch.randn(b, r * world, k, generator=gen)
        # with SP every rank holds its sequence chunk; without it the whole (replicated) sequence
        x_shard = (x_full[:, rank * r:(rank + 1) * r] if sp else x_full).to(dev).bfloat16()
        g_shard = (g_full[:, rank * r:(rank + 1) * r] if sp else g_full).to(dev).bfloat16()
        results = {}
        for fused in (True, False):
            ctx.fused_tensor_collectives = fused
            for prm in list(col.parameters()) + list(row.parameters()):
                prm.grad = None
            x = x_shard.clone().requires_grad_(True)
            h = col(x)
            y = row(h)
            y.backward(g_shard)
            torch.cuda.synchronize()
            results[fused] = {"y": y.detach().float().cpu(), "h": h.detach().float().cpu(), "dx": x.grad.float().cpu(),
                              "dw_col": col.weight.grad.float().cpu(), "db_col": col.bias.grad.float().cpu(),
                              "dw_row": row.weight.grad.float().cpu()}
        from hybrid_training.ops import extension

        errs = {key: float((results[True][key] - results[False][key]).norm() / (results[False][key].norm() + 1e-12))
                for key in results[True]}
        return {"errors": errs, "error_word": int(extension().gemm_error_word(x_shard).abs().sum())}
    finally:
        ctx.shutdown()


def _llama_experiment(world: int, topology: dict[str, Any], *, fused_tp: bool = True, steps: int = 3) -> dict[str, Any]:
    return {"name": "multigpu-llama", "backend": "nccl", "device": "cuda", "timeout_seconds": 120.0,
            "topology": topology,
            "tensor_parallel": {"sequence_parallel": topology.get("sequence_parallel_mode") == "tensor_group",
                                "fused_collectives": fused_tp},
            "model": {"kind": "transformer", "hidden_size": 256, "num_layers": 2, "num_heads": 4, "num_kv_heads": 2,
                      "ffn_hidden_size": 512, "vocab_size": 1024, "max_sequence_length": 256, "norm": "rmsnorm",
                      "position_embedding": "rope", "activation": "swiglu", "bias": False},
            "data": {"micro_batch_size": 2, "sequence_length": 256, "num_train_samples": 4096, "num_eval_samples": 0,
                     "shuffle": False},
            "optimizer": {"learning_rate": 1e-3},
            "mixed_precision": {"enabled": True, "param_dtype": "bfloat16"},
            "fsdp": {"auto_wrap_min_num_params": 10000},
            "training": {"max_steps": steps, "log_every_steps": 0}}


def llama_cuda_worker(rank: int, world: int, topology: dict[str, Any], fused_tp: bool, steps: int) -> dict[str, Any]:
    """A few engine steps of a Llama-style decoder on CUDA under the given topology."""
    cfg = ExperimentConfig.from_dict(_llama_experiment(world, topology, fused_tp=fused_tp, steps=steps))
    ctx = init_distributed(cfg)
    try:
        engine = TrainingEngine(cfg, ctx)
        engine.train(max_steps=steps)
        full = engine.model.full_state_dict()
        out = {"losses": [m.loss for m in engine.history],
               "full": {k: v.detach().float().cpu().clone() for k, v in full.items()}}
        engine.close()
        return out
    finally:
        ctx.shutdown()


def _fsdp_experiment(world: int, *, fused_update: bool, steps: int = 3, accumulation: int = 1,
                     replicas: int = 1) -> dict[str, Any]:
    topology = {"shard_parallel_size": world // replicas}
    if replicas > 1:
        topology["data_parallel_size"] = replicas  # hybrid sharding
    cfg = _llama_experiment(world, topology, steps=steps)
    cfg["fsdp"] = {"auto_wrap_min_num_params": 10000, "fused_update": fused_update}
    cfg["training"] = {"max_steps": steps, "log_every_steps": 0, "gradient_accumulation_steps": accumulation}
    cfg["optimizer"] = {"learning_rate": 1e-3, "weight_decay": 0.1}
    return cfg


def fsdp_fused_kernels_worker(rank: int, world: int) -> dict[str, Any]:
    """The FSDP reduce-scatter + AdamW kernel and the P2P shard all-gather against NCCL + PyTorch AdamW."""
    import torch.distributed as dist

    from hybrid_training.ops import reference_adamw
    from hybrid_training.ops.comm import fsdp_all_gather, fsdp_reduce_scatter_adamw

    cfg = ExperimentConfig.from_dict(_fsdp_experiment(world, fused_update=True))
    ctx = init_distributed(cfg)
    try:
        ws = ctx.symmetric_workspace("shard")
        assert ws is not None, "symmetric memory is unavailable"
        pg = ctx.group("shard").process_group
        dev = ctx.device
        errors: dict[str, float] = {}
        lr, b1, b2, eps, wd, step = 1e-3, 0.9, 0.95, 1e-8, 0.1, 3
        # (shard, non-padding elements of this rank's shard, staging dtype): vector and scalar paths
        for shard, pad, dtype in ((1_000_008, 0, torch.bfloat16), (262_144, 7, torch.float32), (12_345, 5, torch.bfloat16)):
            tag = f"{shard}-{str(dtype)[6:]}"
            gen = torch.Generator(device="cuda").manual_seed(10 + rank)
            staging = ws.allocate(world * shard + 16, dtype)
            staging.copy_(torch.randn(staging.numel(), device=dev, generator=gen).to(dtype))
            total = world * shard - pad
            valid = max(0, min(shard, total - rank * shard))
            # expected gradient: fp32 reduce-scatter of the staged values, averaged, padding zeroed
            full = staging[:world * shard].float().clone()
            expect = torch.empty(shard, device=dev)
            dist.reduce_scatter_tensor(expect, full, group=pg)
            expect /= world
            expect[valid:] = 0
            pgen = torch.Generator(device="cuda").manual_seed(1000)  # same master values on every rank's slot
            param = torch.randn(world * shard, device=dev, generator=pgen)[rank * shard:(rank + 1) * shard].clone()
            m = 0.01 * torch.randn(shard, device=dev, generator=gen)
            v = 0.01 * torch.rand(shard, device=dev, generator=gen)
            ref_p, ref_m, ref_v = param.clone(), m.clone(), v.clone()
            reference_adamw(ref_p, expect, ref_m, ref_v, lr=lr, beta1=b1, beta2=b2, eps=eps, weight_decay=wd, step=step)
            shard16 = ws.allocate(shard, torch.bfloat16)
            hyper = torch.tensor([lr, float(step), 1.0, 0.0], device=dev)
            grad_out = torch.full((shard,), float("nan"), device=dev)
            for _ in range(2):  # the second call checks that the barriers leave the signal pads reusable
                p_run, m_run, v_run = param.clone(), m.clone(), v.clone()
                fsdp_reduce_scatter_adamw(ws, staging, shard16, shard=shard, valid=valid, scale=1.0 / world, param=p_run,
                                          exp_avg=m_run, exp_avg_sq=v_run, hyper=hyper, betas=(b1, b2), eps=eps,
                                          weight_decay=wd, grad_out=grad_out)
            torch.cuda.synchronize()
            ws.check_status()
            scale = float(expect.abs().max()) + 1e-12
            errors[f"grad {tag}"] = float((grad_out - expect).abs().max()) / scale
            errors[f"param {tag}"] = float((p_run - ref_p).abs().max())
            errors[f"exp_avg {tag}"] = float((m_run - ref_m).abs().max())
            errors[f"exp_avg_sq {tag}"] = float((v_run - ref_v).abs().max())
            errors[f"bf16 copy {tag}"] = float((shard16.float() - p_run.bfloat16().float()).abs().max())
            dist.barrier(group=pg)
            out = torch.full((world * shard,), float("nan"), device=dev, dtype=torch.bfloat16)
            fsdp_all_gather(ws, shard16, out)
            expect_full = torch.empty(world * shard, device=dev, dtype=torch.bfloat16)
            dist.all_gather_into_tensor(expect_full, shard16, group=pg)
            torch.cuda.synchronize()
            errors[f"all_gather {tag}"] = 0.0 if torch.equal(out, expect_full) else float("inf")
            dist.barrier(group=pg)
        return {"errors": errors}
    finally:
        ctx.shutdown()


def fsdp_fused_update_worker(rank: int, world: int, fused: bool, steps: int, accumulation: int,
                             replicas: int = 1) -> dict[str, Any]:
    """Engine steps of a Llama-style decoder under FSDP (``replicas`` > 1: hybrid sharding) with or without
    the fused reduce-scatter + AdamW."""
    cfg = ExperimentConfig.from_dict(_fsdp_experiment(world, fused_update=fused, steps=steps, accumulation=accumulation,
                                                      replicas=replicas))
    ctx = init_distributed(cfg)
    try:
        engine = TrainingEngine(cfg, ctx)
        engine.train(max_steps=steps)
        full = engine.model.full_state_dict()
        out = {"fused": engine.fsdp_fused_update, "losses": [m.loss for m in engine.history],
               "full": {k: v.detach().float().cpu().clone() for k, v in full.items()}}
        engine.close()
        return out
    finally:
        ctx.shutdown()


def instrumented_engine_worker(rank: int, world: int, overrides: dict[str, Any], steps: int) -> dict[str, Any]:
    """Train ``steps`` steps through the engine and count every collective of the last one.

    Returns per-step ``{op/group: (calls, bytes)}``, the FSDP memory summary (or ``None``), the
    local parameter / gradient / optimizer-state element counts and the losses.
    """
    from hybrid_training.distributed.collectives import observe_collectives

    cfg = ExperimentConfig.from_dict(overrides)
    ctx = init_distributed(cfg)
    try:
        engine = TrainingEngine(cfg, ctx)
        engine.train(max_steps=steps - 1)
        batches = engine.batch_stream()
        with observe_collectives() as rec:
            engine.history.append(engine.train_step(batches))
        comm = {k: (v.calls, v.bytes) for k, v in rec.by_operation.items()}
        fsdp = engine.model.fsdp
        params = list(engine.model.optimizer_parameters())
        state = engine.optimizer.inner.state
        opt_elems = sum(t.numel() for p in params for t in state.get(p, {}).values() if torch.is_tensor(t) and t.dim() > 0)
        out = {"comm": comm, "memory": fsdp.memory_summary() if fsdp is not None else None,
               "local_params": sum(p.numel() for p in params), "optimizer_elements": opt_elems,
               "grad_elements": sum(p.grad.numel() for p in params if p.grad is not None),
               "losses": [m.loss for m in engine.history],
               "largest_unit": max((u.handle.total_numel for u in fsdp.fsdp_units() if u.handle is not None), default=0)
               if fsdp is not None else 0}
        engine.close()
        return out
    finally:
        ctx.shutdown()


def checkpoint_write_failure_worker(rank: int, world: int, root: str) -> dict[str, Any]:
    """Rank 1's payload write fails (its torch.save raises); every rank must raise the same voted error."""
    from hybrid_training.checkpoint import writer
    from hybrid_training.errors import CheckpointError

    cfg = ExperimentConfig.from_dict({"backend": "gloo", "device": "cpu", "topology": {"shard_parallel_size": world},
                                      "model": {"kind": "mlp", "input_size": 16, "hidden_size": 32, "num_layers": 2,
                                                "output_size": 1},
                                      "data": {"micro_batch_size": 4, "num_train_samples": 64, "num_eval_samples": 0},
                                      "training": {"max_steps": 1, "log_every_steps": 0}})
    ctx = init_distributed(cfg)
    try:
        engine = TrainingEngine(cfg, ctx)
        engine.train(max_steps=1)
        if rank == 1:
            def broken_save(obj: Any, f: Any) -> None:
                raise OSError("no space left on device (injected)")

            writer.torch.save = broken_save  # type: ignore[assignment]
        try:
            engine.save_checkpoint(root)
            return {"raised": False, "message": ""}
        except CheckpointError as exc:
            return {"raised": True, "message": str(exc)}
        finally:
            engine.close()
    finally:
        ctx.shutdown()
