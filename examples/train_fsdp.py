"""Fully sharded data parallelism: each rank keeps 1/N of every flat parameter.

Prints the FSDP units (flat-parameter sizes, this rank's shard, the padding that makes the
flat buffer divisible by the shard count) and the memory held per rank against an unsharded
replica, trains, and then gathers the full parameters once with ``summon_full_params`` to show
that every rank sees the same model.

Run, e.g.: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node N examples/train_fsdp.py --config configs/fsdp_2gpu.yaml`
"""

from __future__ import annotations

from typing import Any

from _common import primary_print, run_training


def show_units(ctx: Any, engine: Any) -> None:
    fsdp = engine.model.fsdp
    if fsdp is None:
        primary_print(ctx, "shard group of one: nothing is sharded")
        return
    rows = [f"{'unit':>4} {'flat numel':>12} {'shard numel':>12} {'padding':>8}"]
    for i, unit in enumerate(u for u in fsdp.fsdp_units() if u.handle is not None):
        h = unit.handle
        rows.append(f"{i:>4} {h.total_numel:>12,} {h.shard_numel:>12,} {h.padding:>8}")
    m = fsdp.memory_summary()
    unsharded = sum(u.handle.total_numel * u.handle.flat_param.element_size() for u in fsdp.fsdp_units() if u.handle is not None)
    fused = "fused reduce-scatter + AdamW kernel" if fsdp.fused_update_enabled else "reduce-scatter, then the optimizer"
    primary_print(ctx, f"FSDP units over {fsdp.shard_group.size} ranks:", *rows,
                  f"per-rank parameter shard {m['shard_bytes']:,} B of {unsharded:,} B unsharded "
                  f"({m['shard_bytes'] / max(unsharded, 1):.1%}); gradient path: {fused}")


def gather_once(ctx: Any, engine: Any) -> None:
    from hybrid_training.distributed.collectives import all_gather_object_in_group

    fsdp = engine.model.fsdp
    if fsdp is None:
        return
    full = engine.model.full_state_dict()  # every unit's shards gathered into full tensors
    total = sum(float(t.double().sum()) for t in full.values())
    sums = all_gather_object_in_group(total, ctx.group("world"))
    name = next(iter(full))
    with fsdp.summon_full_params():  # the module's own attributes are full-size views while inside
        obj: Any = fsdp.module
        for part in name.split("."):
            obj = obj[int(part)] if part.isdigit() else getattr(obj, part)
        shape = tuple(obj.shape)
    primary_print(ctx, f"inside summon_full_params {name} has its full shape {shape}",
                  f"full-parameter checksum on each rank: {sums} -> " + ("identical" if len(set(sums)) == 1 else "MISMATCH"))


if __name__ == "__main__":
    run_training("Fully sharded data parallel", "fsdp_2gpu.yaml", before=show_units, after=gather_once)
