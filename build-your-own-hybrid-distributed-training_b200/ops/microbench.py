"""Micro-benchmarks of the native kernels (CUDA-event timed, warm-up first).

Single GPU::

    python -m hybrid_training.ops.microbench gemm [--only NAME] [--iters N]
    python -m hybrid_training.ops.microbench attention [--shape gpt2|llama8b] [--once]
    python -m hybrid_training.ops.microbench norm [--once]
    python -m hybrid_training.ops.microbench mlp [--rows 8192 --hidden 2048 --ffn 5504]

Several GPUs (one process per GPU, e.g. ``torchrun --nproc-per-node 2 --master-addr 127.0.0.1``)::

    python -m hybrid_training.ops.microbench tp-layer [--seq 4096]
    python -m hybrid_training.ops.microbench allreduce [--mb 154]
    python -m hybrid_training.ops.microbench fsdp [--numel 50597888]

``--once`` launches each kernel a fixed small number of times without timing, which is the
form to run under a profiler.  Each timed line reports the median of the timed iterations and
the achieved rate; between GEMM iterations a 256 MB buffer is rewritten so that operands come
from HBM rather than the 126 MB L2.
"""

from __future__ import annotations

import argparse
import math
import os
import sys
from collections.abc import Callable

import torch

GEMM_SHAPES = {  # name: (M, N, K, A MN-major, B MN-major, fp32 accumulate output)
    "qkv": (8192, 2304, 768, False, False, False),
    "fc1": (8192, 3072, 768, False, False, False),
    "fc2": (8192, 768, 3072, False, False, False),
    "head": (8192, 50257, 768, False, False, False),
    "dgrad_fc2": (8192, 3072, 768, False, True, False),
    "dgrad_head": (8192, 768, 50257, False, True, False),
    "wgrad_fc1": (3072, 768, 8192, True, True, True),
    "wgrad_head": (50257, 768, 8192, True, True, True),
    "square_8k": (8192, 8192, 8192, False, False, False),
}


def _time(fn: Callable[[], None], iters: int, flush: torch.Tensor | None = None) -> float:
    """Median milliseconds of ``fn`` over ``iters`` timed launches after three warm-up calls."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        stop.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(stop))
    times.sort()
    return times[len(times) // 2]


def _padded(t: torch.Tensor) -> torch.Tensor:
    """``t`` with rows padded to 16 bytes (the TMA row-stride rule), as the framework stores them."""
    if (t.stride(0) * 2) % 16 == 0:
        return t
    cols = (t.shape[1] + 7) // 8 * 8
    return torch.zeros(t.shape[0], cols, dtype=t.dtype, device=t.device)[:, : t.shape[1]].copy_(t)


def bench_gemm(only: str | None, iters: int, extra: list[str] | None = None) -> None:
    """``extra`` adds shapes written ``M,N,K[,a_mn,b_mn,f32]`` (0/1 flags), e.g. ``32768,768,3072``."""
    from . import gemm

    dev = torch.device("cuda")
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    shapes = dict(GEMM_SHAPES)
    for spec in extra or []:
        v = [int(t) for t in spec.split(",")]
        v += [0] * (6 - len(v))
        shapes[spec] = (v[0], v[1], v[2], bool(v[3]), bool(v[4]), bool(v[5]))
        only = only if only is not None else "__extra__"
    for name, (m, n, k, amn, bmn, f32) in shapes.items():
        if only == "__extra__":
            if name in GEMM_SHAPES:
                continue
        elif only and name != only:
            continue
        a = _padded(torch.randn((k, m) if amn else (m, k), device=dev).bfloat16())
        b = _padded(torch.randn((k, n) if bmn else (n, k), device=dev).bfloat16())
        out = torch.zeros(m, (n + 63) // 64 * 64, device=dev, dtype=torch.float32 if f32 else torch.bfloat16)[:, :n]
        from ._ext import extension

        extension().set_gemm_pair(1)
        pair = _time(lambda: gemm(a, b, out=out, a_mn_major=amn, b_mn_major=bmn, beta=1.0 if f32 else 0.0), iters, flush)
        extension().set_gemm_pair(0)
        ours = _time(lambda: gemm(a, b, out=out, a_mn_major=amn, b_mn_major=bmn, beta=1.0 if f32 else 0.0), iters, flush)
        aa, bb = (a.t() if amn else a), (b if bmn else b.t())
        lib = _time(lambda: torch.matmul(aa, bb), iters, flush)
        flops = 2.0 * m * n * k
        print(f"gemm {name:11s} M={m} N={n} K={k}: {ours * 1e3:8.1f} us {flops / ours / 1e9:7.1f} TFLOP/s "
              f"(CTA-pair tiles {pair * 1e3:7.1f} us {flops / pair / 1e9:7.1f}) | "
              f"torch.matmul {lib * 1e3:8.1f} us {flops / lib / 1e9:7.1f} TFLOP/s", flush=True)


ATTN_SHAPES = {"gpt2": (8, 1024, 12, 12, 64), "llama8b": (1, 4096, 32, 8, 128)}


def bench_attention(shape: str, once: bool, fast: bool = False) -> None:
    """``fast``: the backward without the reproducibility requirement (one fused kernel at D = 64)."""
    from ._ext import extension

    ext = extension()
    ext.set_deterministic_reductions(not fast)
    dev = torch.device("cuda")
    b, s, h, hkv, d = ATTN_SHAPES[shape]
    scale = 1.0 / math.sqrt(d)
    qkv = (torch.randn(b, s, (h + 2 * hkv) * d, device=dev) * 0.5).bfloat16()
    out = torch.empty(b, s, h * d, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(b, h, s, device=dev)
    dout = torch.randn_like(out)
    dqkv = torch.empty_like(qkv)
    delta = torch.empty(b, h, s, device=dev)
    fwd = lambda: ext.attention_forward(qkv, out, lse, h, hkv, d, True, scale)  # noqa: E731
    bwd = lambda: ext.attention_backward(qkv, out, dout, lse, delta, dqkv, h, hkv, d, True, scale)  # noqa: E731
    if once:
        fwd(), fwd(), bwd(), bwd()
        torch.cuda.synchronize()
        print("attention: launched", flush=True)
        return
    flops = 4.0 * b * h * s * s * d / 2  # causal
    tf, tb = _time(fwd, 10), _time(bwd, 10)
    print(f"attention {shape}{' (fast backward)' if fast else ''} B={b} S={s} H={h} Hkv={hkv} D={d}: forward {tf * 1e3:.1f} us ({flops / tf / 1e9:.0f} TFLOP/s), "
          f"backward {tb * 1e3:.1f} us ({2.5 * flops / tb / 1e9:.0f} TFLOP/s)", flush=True)


def bench_norm(once: bool) -> None:
    from ._ext import extension

    ext = extension()
    dev = torch.device("cuda")
    rows, d = 8192, 768
    res = torch.randn(rows, d, device=dev)
    delta = torch.randn(rows, d, device=dev).bfloat16()
    w, bias = torch.ones(d, device=dev), torch.zeros(d, device=dev)
    r, y = torch.empty(rows, d, device=dev), torch.empty(rows, d, device=dev, dtype=torch.bfloat16)
    mean, rstd = torch.empty(rows, device=dev), torch.empty(rows, device=dev)
    dy, dr = torch.randn(rows, d, device=dev).bfloat16(), torch.randn(rows, d, device=dev)
    dres, ddelta = torch.empty(rows, d, device=dev), torch.empty(rows, d, device=dev, dtype=torch.bfloat16)
    blocks = ext.norm_backward_blocks(rows)
    pw, pb = torch.empty(blocks, d, device=dev), torch.empty(blocks, d, device=dev)
    fwd = lambda: ext.norm_forward(res, delta, w, bias, r, y, mean, rstd, 1e-5, False)  # noqa: E731
    bwd = lambda: ext.norm_backward(dy, dr, r, w, mean, rstd, dres, ddelta, pw, pb, False)  # noqa: E731
    if once:
        fwd(), fwd(), bwd(), bwd()
        torch.cuda.synchronize()
        print("norm: launched", flush=True)
        return
    tf, tb = _time(fwd, 20), _time(bwd, 20)
    fwd_bytes = rows * d * (4 + 2 + 4 + 2)
    bwd_bytes = rows * d * (2 + 4 + 4 + 4 + 2)
    print(f"layernorm rows={rows} d={d}: forward {tf * 1e3:.1f} us ({fwd_bytes / tf / 1e6:.0f} GB/s), "
          f"backward {tb * 1e3:.1f} us ({bwd_bytes / tb / 1e6:.0f} GB/s)", flush=True)


def bench_mlp(rows: int, hidden: int, ffn: int) -> None:
    """SwiGLU MLP forward + backward: activation in the GEMM epilogues vs GEMMs plus element-wise kernels."""
    from .linear import gemm, swiglu, swiglu_mlp

    dev = torch.device("cuda")
    x = torch.randn(rows, hidden, device=dev).bfloat16().requires_grad_(True)
    w1 = (torch.randn(2 * ffn, hidden, device=dev) * 0.02).bfloat16().requires_grad_(True)
    w2 = (torch.randn(hidden, ffn, device=dev) * 0.02).bfloat16().requires_grad_(True)
    g = torch.randn(rows, hidden, device=dev).bfloat16()

    def fused() -> None:
        swiglu_mlp(x, w1, None, w2, None).backward(g)

    def unfused() -> None:
        h = gemm(x.detach(), w1.detach())
        hh = h.requires_grad_(True)
        a = swiglu(hh)
        y = gemm(a.detach(), w2.detach())
        da = gemm(g, w2.detach(), b_mn_major=True)
        a.backward(da)
        dh = hh.grad
        gemm(dh, w1.detach(), b_mn_major=True)
        gemm(dh, x.detach(), a_mn_major=True, b_mn_major=True)
        gemm(g, a.detach(), a_mn_major=True, b_mn_major=True)
        del y

    flops = 2 * rows * hidden * 3 * ffn * 3  # three GEMMs of the forward, twice that in the backward
    tf, tu = _time(fused, 10), _time(unfused, 10)
    print(f"swiglu mlp rows={rows} hidden={hidden} ffn={ffn}: fused {tf * 1e3:.0f} us ({flops / tf / 1e9:.0f} TFLOP/s), "
          f"GEMMs + element-wise {tu * 1e3:.0f} us ({flops / tu / 1e9:.0f} TFLOP/s)", flush=True)


def _init_group(kind: str, hidden: int, seq: int):  # noqa: ANN202
    from ..config import ExperimentConfig
    from ..distributed import init_distributed

    world = int(os.environ.get("WORLD_SIZE", "1"))
    topo = ({"tensor_parallel_size": world, "sequence_parallel_mode": "tensor_group"} if kind == "tp"
            else {"data_parallel_size": world})
    cfg = ExperimentConfig.from_dict({
        "name": "microbench", "backend": "nccl", "device": "cuda", "timeout_seconds": 120.0, "topology": topo,
        "tensor_parallel": {"sequence_parallel": kind == "tp", "fused_collectives": True},
        "mixed_precision": {"enabled": True, "param_dtype": "bfloat16"},
        "model": {"kind": "transformer", "hidden_size": hidden, "num_layers": 1, "num_heads": 32, "vocab_size": 512,
                  "max_sequence_length": seq}})
    return init_distributed(cfg), world


def _max_over_ranks(ms: float) -> float:
    import torch.distributed as dist

    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=dist.group.WORLD)
    return float(t)


def bench_tp_layer(seq: int) -> None:
    """Llama-3-8B-shape MLP + attention projections under TP+SP: fused collective GEMMs vs NCCL."""
    import torch.distributed as dist

    from ..parallel.tensor_parallel import ColumnParallelLinear, RowParallelLinear

    ctx, world = _init_group("tp", 4096, seq)
    try:
        g, dev, d = ctx.group("tensor"), ctx.device, 4096
        qkv = ColumnParallelLinear(d, 6144, g, bias=False, sequence_parallel=True, device=dev)
        proj = RowParallelLinear(4096, d, g, bias=False, sequence_parallel=True, device=dev)
        up = ColumnParallelLinear(d, 28672, g, bias=False, sequence_parallel=True, device=dev)
        down = RowParallelLinear(14336, d, g, bias=False, sequence_parallel=True, device=dev)
        x = torch.randn(1, seq // world, d, device=dev).bfloat16()

        def layer() -> None:
            xx = x.clone().requires_grad_(True)
            o = proj(qkv(xx)[..., : 4096 // world].contiguous())
            y = down(up(o)[..., : 14336 // world].contiguous())
            y.backward(torch.ones_like(y))

        result = {}
        for fused in (True, False):
            ctx.fused_tensor_collectives = fused
            dist.barrier(group=dist.group.WORLD)
            result[fused] = _max_over_ranks(_time(layer, 5))
        flops = 6.0 * seq * d * (6144 + 4096 + 28672 + 14336) / world
        if ctx.rank == 0:
            print(f"tp-layer TP{world} S={seq}: fused {result[True]:.3f} ms ({flops / result[True] / 1e9:.0f} TFLOP/s per GPU), "
                  f"NCCL {result[False]:.3f} ms ({flops / result[False] / 1e9:.0f} TFLOP/s per GPU)", flush=True)
    finally:
        ctx.shutdown()


def bench_allreduce(mb: float) -> None:
    """In-kernel NVLink bucket all-reduce (average) against NCCL on the same fp32 buffer."""
    import torch.distributed as dist

    from .comm import bucket_all_reduce

    ctx, world = _init_group("dp", 256, 256)
    try:
        ws = ctx.symmetric_workspace("data_parallel")
        n = int(mb * 1024 * 1024 / 4) // 4 * 4
        flat = ws.allocate(n, torch.float32)
        flat.normal_()
        pg = ctx.group("data_parallel").process_group
        wide = _max_over_ranks(_time(lambda: bucket_all_reduce(ws, flat, 0, n, 1.0 / world, wide=True), 10))
        narrow = _max_over_ranks(_time(lambda: bucket_all_reduce(ws, flat, 0, n, 1.0 / world, wide=False), 10))
        nccl = _max_over_ranks(_time(lambda: dist.all_reduce(flat, group=pg), 10))
        ws.check_status()
        bus = 2.0 * (world - 1) / world * n * 4  # bytes each rank moves in a ring all-reduce
        if ctx.rank == 0:
            print(f"allreduce {world} ranks {mb:.0f} MB fp32: in-kernel wide {wide * 1e3:.1f} us ({bus / wide / 1e6:.0f} GB/s bus), "
                  f"narrow (co-resident shape) {narrow * 1e3:.1f} us ({bus / narrow / 1e6:.0f} GB/s bus), "
                  f"NCCL {nccl * 1e3:.1f} us ({bus / nccl / 1e6:.0f} GB/s bus)", flush=True)
    finally:
        ctx.shutdown()


def bench_fsdp(numel: int) -> None:
    """FSDP unit of ``numel`` parameters: fused reduce-scatter + AdamW and P2P all-gather against NCCL.

    Baseline gradient path: bf16 gradient cast to fp32, NCCL reduce-scatter (average), fused AdamW
    kernel on the fp32 shard.  Fused path: bf16 gradient copied into the peer-mapped staging buffer,
    then one kernel.  All-gather: NCCL ``all_gather_into_tensor`` of the bf16 shard, the P2P kernel,
    and one copy-engine ``cudaMemcpyAsync`` per peer from the peer-mapped shard.
    """
    import torch.distributed as dist

    from .comm import fsdp_all_gather, fsdp_reduce_scatter_adamw
    from .optim import adamw_flat

    ctx, world = _init_group("dp", 256, 256)
    try:
        ws = ctx.symmetric_workspace("data_parallel")
        pg = ctx.group("data_parallel").process_group
        shard = -(-numel // world // 8) * 8
        padded = shard * world
        dev = ctx.device
        grad = torch.randn(padded, device=dev).bfloat16()
        staging = ws.allocate(padded, torch.bfloat16)
        shard16 = ws.allocate(shard, torch.bfloat16)
        param, m, v = torch.randn(shard, device=dev), torch.zeros(shard, device=dev), torch.zeros(shard, device=dev)
        hyper = torch.tensor([1e-4, 1.0, 1.0, 0.0], device=dev)
        g32 = torch.empty(shard, device=dev)
        copy16 = torch.empty(shard, device=dev, dtype=torch.bfloat16)

        def fused() -> None:
            staging.copy_(grad)
            fsdp_reduce_scatter_adamw(ws, staging, shard16, shard=shard, valid=shard, scale=1.0 / world, param=param,
                                      exp_avg=m, exp_avg_sq=v, hyper=hyper, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)

        def baseline() -> None:
            full = grad.float()
            full.div_(world)
            dist.reduce_scatter_tensor(g32, full, group=pg)
            adamw_flat(param, g32, m, v, copy16, hyper, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1)

        out = torch.empty(padded, device=dev, dtype=torch.bfloat16)

        def copy_engine() -> None:
            fsdp_all_gather(ws, shard16, out, copy_engine=True)

        dist.barrier(group=dist.group.WORLD)
        t_fused = _max_over_ranks(_time(fused, 10))
        t_base = _max_over_ranks(_time(baseline, 10))
        t_ag_p2p = _max_over_ranks(_time(lambda: fsdp_all_gather(ws, shard16, out), 10))
        t_ag_ce = _max_over_ranks(_time(copy_engine, 10))
        t_ag_nccl = _max_over_ranks(_time(lambda: dist.all_gather_into_tensor(out, shard16, group=pg), 10))
        ws.check_status()
        remote = (world - 1) / world * padded * 2  # bf16 bytes each rank reads over NVLink
        if ctx.rank == 0:
            print(f"fsdp unit {numel / 1e6:.1f}M params, {world} ranks: reduce-scatter + AdamW fused {t_fused * 1e3:.1f} us "
                  f"(NVLink {remote / t_fused / 1e6:.0f} GB/s per rank), NCCL + AdamW kernel {t_base * 1e3:.1f} us", flush=True)
            print(f"fsdp unit all-gather bf16: P2P kernel {t_ag_p2p * 1e3:.1f} us ({remote / t_ag_p2p / 1e6:.0f} GB/s), "
                  f"copy engine {t_ag_ce * 1e3:.1f} us ({remote / t_ag_ce / 1e6:.0f} GB/s), NCCL {t_ag_nccl * 1e3:.1f} us "
                  f"({remote / t_ag_nccl / 1e6:.0f} GB/s)", flush=True)
    finally:
        ctx.shutdown()


def main(argv: list[str] | None = None) -> None:
    p = argparse.ArgumentParser(description="Native kernel micro-benchmarks")
    sub = p.add_subparsers(dest="what", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--only", choices=list(GEMM_SHAPES))
    g.add_argument("--iters", type=int, default=20)
    g.add_argument("--shape", action="append", default=[], help="extra shape M,N,K[,a_mn,b_mn,f32]; only these run")
    a = sub.add_parser("attention")
    a.add_argument("--shape", choices=list(ATTN_SHAPES), default="gpt2")
    a.add_argument("--once", action="store_true")
    a.add_argument("--fast", action="store_true", help="backward without the reproducibility requirement")
    n = sub.add_parser("norm")
    n.add_argument("--once", action="store_true")
    ml = sub.add_parser("mlp")
    ml.add_argument("--rows", type=int, default=8192)
    ml.add_argument("--hidden", type=int, default=2048)
    ml.add_argument("--ffn", type=int, default=5504)
    t = sub.add_parser("tp-layer")
    t.add_argument("--seq", type=int, default=4096)
    r = sub.add_parser("allreduce")
    r.add_argument("--mb", type=float, default=154.0)
    f = sub.add_parser("fsdp")
    f.add_argument("--numel", type=int, default=50_597_888)
    args = p.parse_args(argv)
    if args.what == "gemm":
        bench_gemm(args.only, args.iters, args.shape)
    elif args.what == "attention":
        bench_attention(args.shape, args.once, args.fast)
    elif args.what == "norm":
        bench_norm(args.once)
    elif args.what == "mlp":
        bench_mlp(args.rows, args.hidden, args.ffn)
    elif args.what == "tp-layer":
        bench_tp_layer(args.seq)
    elif args.what == "fsdp":
        bench_fsdp(args.numel)
    else:
        bench_allreduce(args.mb)


if __name__ == "__main__":
    main(sys.argv[1:])
