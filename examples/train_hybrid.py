"""Full 4-D hybrid grid: data-parallel replicas x FSDP shards x sequence x tensor parallelism.

Prints every rank's coordinates in the grid and the ranks it shares each process group with
(gathered from all ranks), then trains; the parallel plan printed before it lists which
collective each phase of the step uses.

Run, e.g.: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node N examples/train_hybrid.py --config configs/hybrid_8gpu.yaml`
"""

from __future__ import annotations

from typing import Any

from _common import primary_print, run_training

GROUPS = ("data_parallel", "shard", "sequence", "tensor")


def show_grid(ctx: Any, engine: Any) -> None:
    from hybrid_training.distributed.collectives import all_gather_object_in_group

    mine = {"rank": ctx.rank, "coords": ctx.coordinates.as_tuple(),
            "groups": {g: list(ctx.group(g).ranks) for g in GROUPS}}
    everyone = all_gather_object_in_group(mine, ctx.group("world"))
    rows = [f"{'rank':>4}  {'(dp, shard, seq, tp)':<22}" + "".join(f" {g:<16}" for g in GROUPS)]
    for r in sorted(everyone, key=lambda x: x["rank"]):
        rows.append(f"{r['rank']:>4}  {str(r['coords']):<22}" + "".join(f" {str(r['groups'][g]):<16}" for g in GROUPS))
    primary_print(ctx, "rank grid (tensor is the fastest-varying dimension, so each tensor group sits on one node):", *rows)


if __name__ == "__main__":
    run_training("Full 4-D hybrid grid", "hybrid_8gpu.yaml", before=show_grid)
