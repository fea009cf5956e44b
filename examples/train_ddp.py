"""Bucketed data parallelism: one replica per rank, gradients all-reduced bucket by bucket.

Prints the bucket plan (which parameters share a bucket, its size, and whether the reduction
runs as the in-kernel NVLink all-reduce over symmetric memory or as an NCCL call), then trains,
then checks that every replica ended with bit-identical parameters and prints the reduction
counters.

Run, e.g.: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node N examples/train_ddp.py --config configs/ddp_2gpu.yaml`
"""

from __future__ import annotations

from typing import Any

from _common import primary_print, run_training


def show_buckets(ctx: Any, engine: Any) -> None:
    ddp = engine.model.ddp
    if ddp is None:
        primary_print(ctx, "one data-parallel rank: the model is not wrapped, nothing is reduced")
        return
    path = ("in-kernel all-reduce over symmetric memory (NVLink peer loads, NVLS where present)"
            if ddp.reduction_path == "in-kernel" else f"{ctx.backend} all-reduce")
    rows = [f"{'bucket':>6} {'tensors':>7} {'MiB':>8}  first .. last parameter"]
    for b in ddp.bucket_layouts():
        mib = b.total_numel * 4 / 2**20
        rows.append(f"{b.index:>6} {len(b.parameter_names):>7} {mib:>8.2f}  {b.parameter_names[0]} .. {b.parameter_names[-1]}")
    primary_print(ctx, f"gradient buckets ({ddp.group.size} replicas, reduction: {path}):", *rows,
                  "buckets are reduced in reverse registration order, as the backward pass produces them")


def check_replicas(ctx: Any, engine: Any) -> None:
    ddp = engine.model.ddp
    if ddp is None:
        return
    ddp.verify_replica_consistency()  # raises if any replica's parameters differ
    primary_print(ctx, "replicas agree bit for bit after training", f"DDP counters: {ddp.statistics.as_dict()}")


if __name__ == "__main__":
    run_training("Bucketed DDP", "ddp_2gpu.yaml", before=show_buckets, after=check_replicas)
