"""Tensor parallelism: each rank of the tensor group holds a slice of every large weight.

Prints, for each parameter, the slice this rank holds, the full shape, and the dimension the
weight is split along (column-parallel layers split the output features, row-parallel layers
the input features, the vocabulary-parallel embedding and head the vocabulary), trains, and then
checks that every parameter that is *not* split (norms, row-parallel biases) is identical on all
ranks of the tensor group.

Run, e.g.: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node N examples/train_tensor_parallel.py --config configs/tensor_parallel_2gpu.yaml`
"""

from __future__ import annotations

from typing import Any

from _common import primary_print, run_training


def _kind(name: str, dim: int | None) -> str:
    if dim is None:
        return "replicated"
    if "embed" in name or "head" in name or "lm_head" in name:
        return "vocabulary-parallel"
    return "column-parallel" if dim == 0 else "row-parallel"


def show_slices(ctx: Any, engine: Any) -> None:
    info = engine.model.parameter_parallel_info()
    tp = ctx.group("tensor").size
    rows = [f"{'parameter':<40} {'local':>16} {'full':>16}  split"]
    for name, item in info.items():
        local = tuple(item.shape)
        full = list(local)
        if item.partition_dim is not None:
            full[item.partition_dim] *= tp
        rows.append(f"{name:<40} {str(local):>16} {str(tuple(full)):>16}  {_kind(name, item.partition_dim)}")
    primary_print(ctx, f"tensor-parallel slices on rank 0 of {tp}:", *rows)


def check_replicated(ctx: Any, engine: Any) -> None:
    from hybrid_training.distributed.collectives import assert_tensor_consistent

    group = ctx.group("tensor")
    if group.size == 1:
        return
    info = engine.model.parameter_parallel_info()
    params = dict(engine.model.wrapped.named_parameters())
    checked = 0
    for name, item in info.items():
        if item.partition_dim is None and name in params:
            assert_tensor_consistent(params[name].data, group, name=name, operation="train_tensor_parallel")
            checked += 1
    primary_print(ctx, f"{checked} replicated parameters agree across the {group.size} tensor-parallel ranks")


if __name__ == "__main__":
    run_training("Tensor parallelism", "tensor_parallel_2gpu.yaml", before=show_slices, after=check_replicated)
