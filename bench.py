#!/usr/bin/env python
"""Headline benchmark: GPT-2-124M-shape data-parallel training throughput on B200.

Config (second entry): 12 layers, d_model 768, 12 heads, vocab
50257 (tied embeddings), sequence 1024, micro-batch 8 per GPU, bf16 compute
with fp32 master weights, AdamW, 25 MB DDP gradient buckets, uniform random
token ids, random-init weights.  One process per GPU; for N > 1 launch with
``python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1
bench.py --gpus N``.

Two arms:

* ``--impl native`` (default): this repository's ``TrainingEngine`` (native
  sm_100a kernels, in-kernel NVLink bucket all-reduce, CUDA-graph step);
* ``--impl reference``: the unmodified reference installed in
  ``baseline/_ref``, driven through its public API (``baseline/reference_harness.py``).

Timing: W untimed warm-up steps, then exactly K steps bracketed by a barrier and
``torch.cuda.synchronize()`` and timed with CUDA events on the launching
stream; the reported time is the max over ranks.  ``value`` runs the step on
batches already resident on the device; ``e2e`` runs the same public
``train_step`` on batches in pinned host memory (host-to-device copy every
step) and reads the loss back to the host every step.  The step's working set
(weights, optimizer state, activations: several GB) exceeds the 126 MB L2, so
no explicit L2 flush is inserted.  SM clocks are sampled with nvidia-smi
during the timed region.  Prints one JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "tokens/sec (device-timed, max over ranks) at 1/2/4/8 B200; exposed comm ms/step"
MODEL_NAME = "GPT-2-124M-shape (12L, d768, 12h, V50257, tied), DDP"
SEQ = 1024
MICRO_BATCH = 8
CONFIGS = {  # name -> (model, micro-batch per replica, sequence, gradient accumulation)
    "gpt2_ddp": (MODEL_NAME, MICRO_BATCH, SEQ, 1),
    "llama_fsdp": ("Llama-style 1.3B (24L, d2048, 16h, SwiGLU 5504, V32000), FSDP full shard", 4, 2048, 1),
    "llama_tp_sp": ("Llama-3-8B shape (32L, d4096, 32q/8kv, ffn 14336, V128256), TP+SP", 1, 4096, 1),
    "llama_hybrid": ("Llama-3-8B shape, DP2 x TP(N/2) + SP", 2, 4096, 4),
}


def _args() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["native", "reference"], default="native")
    p.add_argument("--no-graph", action="store_true", help="native arm: run eagerly instead of replaying a CUDA graph")
    p.add_argument("--overlap-step", action="store_true",
                   help="native arm: run the optimizer update bucket by bucket during the backward pass (default: after it)")
    p.add_argument("--config", choices=list(CONFIGS), default="gpt2_ddp",
                   help="gpt2_ddp (the headline, default); llama_fsdp (1.3B full shard, S2048, 4/GPU); llama_tp_sp "
                        "(Llama-3-8B, TP=N with SP, S4096, micro-batch 1); llama_hybrid (Llama-3-8B, DP2 x TP N/2 with SP, "
                        "S4096, global batch 16 by accumulation)")
    return p.parse_args()


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]) -> None:
        self.gpus = set(gpus)
        self.rows: list[list[str]] = []
        self._proc: subprocess.Popen | None = None
        self._thread: threading.Thread | None = None

    def start(self) -> None:
        try:
            self._proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"],
                                          stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None
            return

        def pump() -> None:
            assert self._proc is not None and self._proc.stdout is not None
            for line in self._proc.stdout:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    self.rows.append(parts)

        self._thread = threading.Thread(target=pump, daemon=True)
        self._thread.start()
        deadline = time.monotonic() + 3.0  # nvidia-smi takes a moment to start: let it begin sampling first
        while not self.rows and time.monotonic() < deadline:
            time.sleep(0.01)
        self.rows.clear()

    def stop(self) -> dict:
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)
        rows = [r for r in self.rows if r[0].isdigit() and int(r[0]) in self.gpus]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for name, flag in zip(names[1:], r[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def _visible_gpu_indices(n: int) -> list[int]:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return [int(x) for x in vis.split(",")][:n]
        except ValueError:
            pass
    return list(range(n))


def _parallelism(config: str, n: int) -> str:
    if config == "gpt2_ddp":
        return f"dp{n}"
    if config == "llama_fsdp":
        return f"fsdp{n}"
    if config == "llama_tp_sp":
        return f"tp{n}+sp"
    tp = max(1, n // 2)
    return f"dp{n // tp}xtp{tp}+sp"


def _emit(result: dict) -> None:
    print(json.dumps(result), flush=True)


def _baseline_value() -> float | None:
    """The reference publishes no throughput for any configuration, so there is no ratio to report."""
    return None


def main() -> None:
    args = _args()
    if args.impl == "reference":
        sys.path[:] = [p for p in sys.path if os.path.abspath(p or ".") != ROOT]
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        sys.path.insert(1, os.path.join(ROOT, "baseline"))
        try:
            import reference_harness  # type: ignore[import-not-found]
        except Exception as exc:  # the reference could not be imported at all
            _emit({"impl": "reference", "unavailable": f"reference import failed: {type(exc).__name__}: {exc}"})
            return
        runner = reference_harness.run
    else:
        sys.path.insert(0, ROOT)
        from hybrid_training.bench_runner import run as runner  # noqa: E402

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    sampler = ClockSampler(_visible_gpu_indices(args.gpus)) if rank == 0 else None
    model_name, micro_batch, seq, accum = CONFIGS[args.config]
    extra = {"config": args.config, "grad_accum": accum}
    if args.impl == "native":
        extra["overlap_step"] = args.overlap_step
    result = runner(steps=args.steps, warmup=args.warmup, micro_batch=micro_batch, seq=seq,
                    use_graph=not args.no_graph, clock_start=(sampler.start if sampler else None),
                    clock_stop=(sampler.stop if sampler else None), **extra)
    if rank == 0:
        n = args.gpus
        tokens_per_step = result.get("tokens_per_step") or n * micro_batch * seq
        tokens = tokens_per_step * args.steps
        value = tokens / (result["device_ms"] / 1000.0)
        e2e = tokens / (result["e2e_ms"] / 1000.0)
        out = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": n,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": result["device_ms"] / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None if _baseline_value() is None else value / _baseline_value(),
            "dtype": "bf16",
            "data": "synthetic: uniform random token ids, random-init weights",
            "config": {"model": model_name, "global_batch": tokens_per_step // seq, "seq_len": seq,
                       "parallelism": _parallelism(args.config, n), "micro_batch_per_replica": micro_batch,
                       "grad_accum": accum, "bucket_cap_mb": 25, "optimizer": "AdamW fp32 master",
                       "l2": "no flush: per-step working set of several GB exceeds the 126 MB L2",
                       "cuda_graph": (not args.no_graph) if args.impl == "native" else False,
                       "optimizer_update": ("bucket by bucket during the backward" if args.overlap_step
                                            else "after the backward") if args.impl == "native" else "after the backward"},
            "clocks": result.get("clocks", {}),
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": result["h2d_bytes_per_step"],
                    "d2h_bytes_per_step": result["d2h_bytes_per_step"], "ms_per_step": result["e2e_ms"] / args.steps},
            "gpu_launches": result.get("gpu_launches", 0),
            "exposed_comm_ms_per_step": result.get("exposed_comm_ms_per_step"),
            "final_loss": result.get("loss"),
            "peak_memory_bytes": result.get("peak_memory_bytes"),
        }
        for key in ("communication_per_step", "parameter_bytes", "master_parameter_bytes", "optimizer_state_bytes"):
            if key in result:
                out[key] = result[key]
        if result.get("shape"):
            out["config"]["reference_shape"] = result["shape"]
        if args.impl == "reference":
            out["impl"] = "reference"
            out.pop("gpu_launches")
        _emit(out)
    if dist.is_initialized():
        dist.barrier(group=dist.group.WORLD)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
