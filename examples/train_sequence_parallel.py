"""Megatron sequence parallelism: tensor parallelism plus a sequence split of the activations
that lie between the tensor-parallel regions (norms, dropout, residual adds).

Prints how the sequence is divided over the tensor group and what that does to the activation
memory held between layers, then trains; the report at the end counts the all-gathers and
reduce-scatters that replace tensor parallelism's all-reduces.

Run, e.g.: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node N examples/train_sequence_parallel.py --config configs/sequence_parallel_2gpu.yaml`
"""

from __future__ import annotations

from typing import Any

from _common import primary_print, run_training


def show_split(ctx: Any, engine: Any) -> None:
    cfg = engine.config
    tp = ctx.group("tensor").size
    seq, batch, d = cfg.data.sequence_length, cfg.data.micro_batch_size, cfg.model.hidden_size
    bytes_per = 2 if cfg.mixed_precision.enabled else 4
    full = batch * seq * d * bytes_per
    mode = cfg.topology.sequence_parallel_mode if cfg.topology.sequence_parallel_enabled else "off"
    local = full // tp if cfg.topology.sequence_parallel_enabled else full
    primary_print(ctx, f"sequence parallelism: {mode}; tensor group of {tp}",
                  f"  tokens per rank between layers: {batch} x {seq // tp if local != full else seq} (of {batch} x {seq})",
                  f"  one hidden-state activation: {local:,} B per rank instead of {full:,} B",
                  "  entering a column-parallel layer: all-gather along the sequence; leaving a row-parallel layer:"
                  " reduce-scatter along the sequence")


if __name__ == "__main__":
    run_training("Megatron sequence parallelism", "sequence_parallel_2gpu.yaml", before=show_split)
