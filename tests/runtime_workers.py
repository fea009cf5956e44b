"""Module-level workers for the runtime tests (collectives, context, launcher faults, TP layers, HSDP, counts).

Each function runs inside a Gloo/CPU rank spawned by ``launch_workers`` and returns plain values or
CPU tensors; many checks share one launch so the suite spawns few process groups.
"""

from __future__ import annotations

import os
import time
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from hybrid_training.config import DDPConfig, FSDPConfig, TopologyConfig
from hybrid_training.distributed import CommunicationRecorder, init_distributed
from hybrid_training.distributed.collectives import (
    ReduceOp,
    all_gather_object_in_group,
    all_gather_tensor,
    all_reduce,
    all_to_all_tensor,
    assert_metadata_consistent,
    assert_tensor_consistent,
    broadcast,
    recv_tensor,
    reduce_scatter_tensor,
    send_tensor,
    sum_scalar,
)
from hybrid_training.errors import CollectiveError, ParameterConsistencyError

from .dist_workers import MLP_CFG, mlp_batch


def _raises(fn: Any, kind: type[BaseException]) -> str:
    try:
        fn()
    except kind as exc:
        return str(exc)
    except Exception as exc:  # noqa: BLE001
        return f"WRONG {type(exc).__name__}: {exc}"
    return "NO ERROR"


def collectives_worker(rank: int, world: int) -> dict[str, Any]:
    """Every wrapper in ``distributed.collectives`` on a dp=2 x tensor=world/2 grid."""
    ctx = init_distributed(TopologyConfig(data_parallel_size=2, tensor_parallel_size=world // 2), backend="gloo", device="cpu")
    try:
        out: dict[str, Any] = {}
        w, tp, dp, seq = ctx.group("world"), ctx.group("tensor"), ctx.group("data_parallel"), ctx.group("sequence")
        rec = CommunicationRecorder()
        base = torch.arange(4, dtype=torch.float32) + 10 * rank
        for op in ReduceOp.ALL:
            t = base.clone()
            all_reduce(t, w, op=op, recorder=rec).wait()
            out[f"all_reduce_{op}"] = t
        t = torch.full((3,), float(rank))
        broadcast(t, tp, source_local_rank=1).wait()
        out["broadcast_from_local1"] = t
        g, work = all_gather_tensor(torch.tensor([[rank, rank]], dtype=torch.float32), w, recorder=rec)
        work.wait()
        out["all_gather"] = g
        x = torch.arange(2 * world, dtype=torch.float32) + rank
        rs, work = reduce_scatter_tensor(x.clone(), w, op=ReduceOp.SUM, recorder=rec)
        work.wait()
        out["reduce_scatter_sum"] = rs
        rs_avg, work = reduce_scatter_tensor(x.clone(), w, op=ReduceOp.AVG)
        work.wait()
        out["reduce_scatter_avg"] = rs_avg
        out["reduce_scatter_indivisible"] = _raises(lambda: reduce_scatter_tensor(torch.zeros(world + 1), w), CollectiveError)
        out["all_to_all"] = all_to_all_tensor(torch.arange(world, dtype=torch.float32) + 100 * rank, w, recorder=rec)
        # ring send/recv inside the tensor group (size >= 2)
        me, n = tp.local_rank, tp.size
        payload = torch.tensor([float(rank)])
        received = torch.zeros(1)
        if me % 2 == 0:
            send_tensor(payload, tp, destination_local_rank=(me + 1) % n)
            recv_tensor(received, tp, source_local_rank=(me - 1) % n)
        else:
            recv_tensor(received, tp, source_local_rank=(me - 1) % n)
            send_tensor(payload, tp, destination_local_rank=(me + 1) % n)
        out["ring_received"] = float(received)
        out["send_to_self"] = _raises(lambda: send_tensor(payload, tp, destination_local_rank=me), CollectiveError)
        out["non_contiguous"] = _raises(lambda: all_reduce(torch.zeros(4, 4).t(), w), CollectiveError)
        out["unknown_op"] = _raises(lambda: all_reduce(torch.zeros(2), w, op="product"), CollectiveError)
        out["bad_source"] = _raises(lambda: broadcast(torch.zeros(2), tp, source_local_rank=n), CollectiveError)
        # trivial group: no communication, identity semantics
        t = base.clone()
        all_reduce(t, seq, op=ReduceOp.AVG, recorder=rec).wait()
        out["trivial_all_reduce_identity"] = torch.equal(t, base)
        g1, _ = all_gather_tensor(base.clone(), seq)
        out["trivial_all_gather_copy"] = torch.equal(g1, base)
        # async work: wait time recorded without bumping the call count; completion hook runs once
        calls_before = rec.by_operation["all_reduce/world"].calls
        t = base.clone()
        work = all_reduce(t, w, async_op=True, recorder=rec)
        work.wait()
        work.wait()
        out["async_calls_delta"] = rec.by_operation["all_reduce/world"].calls - calls_before
        out["recorder_keys"] = sorted(rec.by_operation)
        out["all_reduce_bytes"] = rec.by_operation["all_reduce/world"].bytes
        # consistency checks raise on every rank
        out["metadata_mismatch"] = _raises(
            lambda: assert_metadata_consistent({"layout": rank == 1}, w, name="layout"), ParameterConsistencyError)
        assert_metadata_consistent({"layout": 1}, w, name="layout")
        out["tensor_mismatch"] = _raises(
            lambda: assert_tensor_consistent(torch.tensor([float(rank == 0)]), dp, name="weights"), ParameterConsistencyError)
        assert_tensor_consistent(torch.ones(3), dp, name="weights")
        out["sum_scalar"] = sum_scalar(float(rank + 1), w, device=torch.device("cpu"))
        out["objects"] = all_gather_object_in_group({"r": rank}, dp)
        return out
    finally:
        ctx.shutdown()


def failing_worker(rank: int, world: int, mode: str) -> str:
    """Host-side fault injection: one rank raises, or one rank never reaches the collective."""
    ctx = init_distributed(TopologyConfig(data_parallel_size=world), backend="gloo", device="cpu", timeout_seconds=20.0)
    try:
        if rank == 1 and mode == "raise":
            raise RuntimeError("injected failure on rank 1")
        if rank == 1 and mode == "silent":
            time.sleep(120)  # never joins the all-reduce below; the launcher's deadline ends the run
        t = torch.ones(1)
        all_reduce(t, ctx.group("world")).wait()
        return f"done {float(t)}"
    finally:
        ctx.shutdown()


def context_worker(rank: int, world: int) -> dict[str, Any]:
    """Double initialisation is refused; the grid coordinates and group memberships are reported."""
    ctx = init_distributed(TopologyConfig(data_parallel_size=2, shard_parallel_size=world // 2), backend="gloo", device="cpu")
    try:
        again = _raises(lambda: init_distributed(TopologyConfig(data_parallel_size=world), backend="gloo", device="cpu"),
                        Exception)
        return {"again": again, "coords": ctx.topology.coordinates_of(rank).label(),
                "dp_shard": list(ctx.group("dp_shard").ranks), "shard": list(ctx.group("shard").ranks),
                "data_parallel": list(ctx.group("data_parallel").ranks)}
    finally:
        ctx.shutdown()


def bad_topology_worker(rank: int, world: int) -> str:
    try:
        init_distributed(TopologyConfig(data_parallel_size=3), backend="gloo", device="cpu")
    except Exception as exc:  # noqa: BLE001
        return f"{type(exc).__name__}: {exc}"
    return "NO ERROR"


def torch_ddp_oracle_worker(rank: int, world: int, steps: int) -> dict[str, Any]:
    """This DDP against PyTorch's own DistributedDataParallel on the same model, data and optimizer."""
    from torch.nn.parallel import DistributedDataParallel as TorchDDP

    from hybrid_training.models import MLP
    from hybrid_training.parallel import DistributedDataParallel

    ctx = init_distributed(TopologyConfig(data_parallel_size=world), backend="gloo", device="cpu")
    try:
        ours = DistributedDataParallel(MLP(MLP_CFG, seed=0), ctx.group("data_parallel"), DDPConfig(bucket_cap_mb=0.001))
        theirs = TorchDDP(MLP(MLP_CFG, seed=0), process_group=ctx.group("data_parallel").process_group)
        opt_a = torch.optim.SGD(ours.parameters(), lr=0.1)
        opt_b = torch.optim.SGD(theirs.parameters(), lr=0.1)
        diffs = []
        for step in range(steps):
            x, y = mlp_batch(step, rank)
            F.mse_loss(ours(x), y).backward()
            ours.finish_gradient_synchronization()
            F.mse_loss(theirs(x), y).backward()
            for (_, pa), (_, pb) in zip(ours.module.named_parameters(), theirs.module.named_parameters()):
                diffs.append(float((pa.grad - pb.grad).abs().max()))
            opt_a.step()
            opt_b.step()
            opt_a.zero_grad()
            opt_b.zero_grad()
        return {"max_grad_diff": max(diffs), "layouts": len(ours.bucket_layouts())}
    finally:
        ctx.shutdown()


def tp_layers_worker(rank: int, world: int) -> dict[str, Any]:
    """Column / row / vocab-parallel layers against full nn.Linear / nn.Embedding (same seeded init)."""
    from hybrid_training.models.transformer import build_reference_linear
    from hybrid_training.parallel import ColumnParallelLinear, RowParallelLinear, VocabParallelEmbedding

    ctx = init_distributed(TopologyConfig(tensor_parallel_size=world), backend="gloo", device="cpu")
    try:
        g = ctx.group("tensor")
        out: dict[str, float] = {}
        x = torch.randn(6, 16, generator=torch.Generator().manual_seed(7), requires_grad=True)
        ref = build_reference_linear(16, 8 * world, bias=True, init_seed=3)
        y_ref = ref(x)
        y_ref.square().sum().backward()
        gx_ref = x.grad.clone()
        x.grad = None
        col = ColumnParallelLinear(16, 8 * world, g, bias=True, gather_output=True, init_seed=3)
        y = col(x)
        y.square().sum().backward()
        out["column_forward"] = float((y - y_ref).abs().max())
        out["column_input_grad"] = float((x.grad - gx_ref).abs().max())
        lo = rank * 8
        out["column_weight_grad"] = float((col.weight.grad - ref.weight.grad[lo:lo + 8]).abs().max())
        out["column_full_weight"] = float((col.full_weight() - ref.weight).abs().max())
        # row-parallel consumes the input split along features
        xr = torch.randn(6, 8 * world, generator=torch.Generator().manual_seed(9))
        ref_r = build_reference_linear(8 * world, 16, bias=True, init_seed=5)
        row = RowParallelLinear(8 * world, 16, g, bias=True, input_is_parallel=True, init_seed=5)
        yr = row(xr[:, lo:lo + 8].contiguous())
        out["row_forward"] = float((yr - ref_r(xr)).abs().max())
        out["row_full_weight"] = float((row.full_weight() - ref_r.weight).abs().max())
        # vocab-parallel embedding
        emb = VocabParallelEmbedding(32 * world, 8, g, init_seed=11)
        ids = torch.randint(0, 32 * world, (3, 5), generator=torch.Generator().manual_seed(1))
        full = emb.full_weight()
        out["embedding_forward"] = float((emb(ids) - F.embedding(ids, full)).abs().max())
        return out
    finally:
        ctx.shutdown()


def hsdp_worker(rank: int, world: int, steps: int) -> dict[str, Any]:
    """Hybrid sharding: shard over pairs, replicate across pairs (dp=2 x shard=2)."""
    from hybrid_training.models import MLP
    from hybrid_training.optim import FusedAdamW
    from hybrid_training.parallel import FullyShardedDataParallel

    ctx = init_distributed(TopologyConfig(data_parallel_size=2, shard_parallel_size=world // 2), backend="gloo", device="cpu")
    try:
        rec = CommunicationRecorder()
        fsdp = FullyShardedDataParallel(MLP(MLP_CFG, seed=0), ctx.group("shard"), FSDPConfig(),
                                        replica_group=ctx.group("data_parallel"), recorder=rec)
        opt = FusedAdamW([fsdp.handle.flat_param], lr=1e-3, weight_decay=0.0)
        data_rank = ctx.group("dp_shard").local_rank
        for step in range(steps):
            x, y = mlp_batch(step, data_rank)
            F.mse_loss(fsdp(x), y).backward()
            fsdp.finish_backward()
            opt.step()
            opt.zero_grad()
        return {"full": fsdp.full_state_dict(), "ops": sorted(rec.by_operation), "data_rank": data_rank}
    finally:
        ctx.shutdown()


def comm_volume_worker(rank: int, world: int, strategy: str, reshard: bool) -> dict[str, Any]:
    """Bytes and calls of one training step: DDP all-reduces the gradients; FSDP all-gathers and reduce-scatters."""
    from hybrid_training.models import MLP
    from hybrid_training.parallel import DistributedDataParallel, FullyShardedDataParallel

    ctx = init_distributed(TopologyConfig(data_parallel_size=world) if strategy == "ddp" else
                           TopologyConfig(shard_parallel_size=world), backend="gloo", device="cpu")
    try:
        rec = CommunicationRecorder()
        model = MLP(MLP_CFG, seed=0)
        n = sum(p.numel() for p in model.parameters())
        if strategy == "ddp":
            wrapped: nn.Module = DistributedDataParallel(model, ctx.group("data_parallel"), DDPConfig(bucket_cap_mb=25.0),
                                                         recorder=rec)
        else:
            wrapped = FullyShardedDataParallel(model, ctx.group("shard"), FSDPConfig(reshard_after_forward=reshard, prefetch=False),
                                               recorder=rec, sync_module_states=False)
        rec.reset()
        x, y = mlp_batch(0, rank)
        F.mse_loss(wrapped(x), y).backward()
        if strategy == "ddp":
            wrapped.finish_gradient_synchronization()
        else:
            wrapped.finish_backward()
        return {"params": n, "ops": {k: (v.calls, v.bytes) for k, v in rec.by_operation.items()},
                "padded": None if strategy == "ddp" else wrapped.handle.padded_numel}
    finally:
        ctx.shutdown()


def env_probe_worker(rank: int, world: int) -> dict[str, str]:
    return {k: os.environ.get(k, "") for k in ("RANK", "WORLD_SIZE", "MASTER_ADDR", "LOCAL_RANK")}


def independent_sp_worker(rank: int, world: int, kind: str, algorithm: str = "all_gather") -> dict[str, Any]:
    """Sequence parallelism over its own grid dimension (``independent`` mode, tensor width 1)."""
    import dataclasses as dc

    from hybrid_training.config import ExperimentConfig
    from hybrid_training.parallel import all_reduce_sequence_parallel_gradients, build_model

    from .dist_workers import _tiny_transformer

    topo = TopologyConfig(sequence_parallel_size=world, sequence_parallel_mode="independent")
    cfg = ExperimentConfig(backend="gloo", device="cpu", topology=topo, model=_tiny_transformer(kind),
                           tensor_parallel=dc.replace(ExperimentConfig().tensor_parallel, sequence_parallel=True,
                                                      context_parallel_algorithm=algorithm))
    ctx = init_distributed(cfg)
    try:
        model = build_model(cfg, ctx)
        tokens = torch.randint(0, 64, (2, 17), generator=torch.Generator().manual_seed(7))
        logits = model(tokens[:, :-1])
        loss = model(tokens[:, :-1], targets=tokens[:, 1:])
        loss.backward()
        all_reduce_sequence_parallel_gradients(model, ctx.group("sequence_effective"))
        grads = {n: p.grad.clone() for n, p in model.named_parameters()
                 if p.grad is not None and ("input_norm.weight" in n or "qkv.weight" in n)}
        return {"loss": float(loss.detach()), "logits": logits.detach().clone(), "grads": grads}
    finally:
        ctx.shutdown()
