"""Llama-shaped models on B200: RMSNorm, rotary positions, SwiGLU, grouped-query attention, under
FSDP (``llama_1b3_fsdp_8gpu.yaml``) or tensor + sequence parallelism (``llama3_8b_tp8_sp.yaml``,
``llama3_8b_hybrid_dp2_tp4.yaml``).

Prints the model shape, the median step time and the achieved model-FLOP rate per GPU.

Run, e.g.: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node N examples/train_llama.py --config configs/llama_1b3_fsdp_8gpu.yaml`
"""

from __future__ import annotations

from typing import Any

from _common import primary_print, run_training


def show_throughput(ctx: Any, engine: Any) -> None:
    cfg = engine.config
    counts = engine.parameter_count()
    m, seq = cfg.model, cfg.data.sequence_length
    per_token = 6 * counts["global"] + 12 * m.num_layers * seq * m.hidden_size  # weights + causal attention (x0.5)
    timed = [h for h in engine.history[1:] if h.seconds > 0] or engine.history
    if not timed:
        return
    seconds = sorted(h.seconds for h in timed)[len(timed) // 2]
    tokens = timed[-1].samples * seq if timed[-1].samples else cfg.data.micro_batch_size * seq * ctx.group("dp_shard").size
    primary_print(ctx, f"model: {m.num_layers} layers, d={m.hidden_size}, {m.num_heads} heads "
                  f"({m.num_kv_heads or m.num_heads} key/value), vocabulary {m.vocab_size}, {counts['global']:,} parameters",
                  f"median step {seconds * 1e3:.2f} ms (host clock, first step excluded): {tokens / seconds:,.0f} tokens/s, "
                  f"{per_token * tokens / seconds / ctx.world_size / 1e12:.1f} TFLOP/s per rank "
                  f"(model FLOPs {per_token / 1e9:.2f} GFLOP/token)")


if __name__ == "__main__":
    run_training("Llama-shaped FSDP / TP+SP on B200", "llama_1b3_fsdp_8gpu.yaml", after=show_throughput)
