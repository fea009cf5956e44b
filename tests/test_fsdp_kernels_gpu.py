"""The FSDP reduce-scatter + AdamW kernel and the shard all-gathers on ONE GPU, peers emulated in local memory.

Both "ranks'" staging buffers and signal pads are ordinary allocations on this device, so the
kernel runs as one rank of a group of two without any second process.  This rank's arrival
flag from the "peer" is set beforehand, so the opening barrier passes at once; nothing can
release the closing barrier, whose bounded wait runs out and reports stage 12 in the status
word, by which time the reduction and the update have been written.  The test checks the
arithmetic (rank-order fp32 sum of bf16 or fp32 gradients, 1/G scale, zeroed padding, AdamW,
bf16 shard copy) against PyTorch on the vector and scalar paths, and both all-gather variants.
The multi-GPU tests run the same kernels across real peers.
"""

from __future__ import annotations

import pytest
import torch

from hybrid_training.ops import reference_adamw

pytestmark = pytest.mark.gpu

_BLOCKS = 148  # upper bound on the kernel's grid (one block per SM)


def _ext():
    import hybrid_training.ops as ops

    return ops.extension()  # fails loudly when the native module is missing


@pytest.mark.parametrize("rank", [0, 1])
@pytest.mark.parametrize("shard,pad,dtype", [(1_000_008, 0, torch.bfloat16), (262_144, 7, torch.float32),
                                             (12_345, 5, torch.bfloat16)])
def test_reduce_scatter_adamw_arithmetic(rank: int, shard: int, pad: int, dtype: torch.dtype) -> None:
    ext = _ext()
    dev = torch.device("cuda")
    world = 2
    gen = torch.Generator(device="cuda").manual_seed(3 + rank)
    staging = [torch.randn(world * shard, device=dev, generator=gen).to(dtype) for _ in range(world)]
    total = world * shard - pad
    valid = max(0, min(shard, total - rank * shard))
    expect = (staging[0][rank * shard:(rank + 1) * shard].float() + staging[1][rank * shard:(rank + 1) * shard].float()) / world
    expect[valid:] = 0
    param = torch.randn(shard, device=dev, generator=gen)
    m = 0.01 * torch.randn(shard, device=dev, generator=gen)
    v = 0.01 * torch.rand(shard, device=dev, generator=gen)
    lr, b1, b2, eps, wd, step = 1e-3, 0.9, 0.95, 1e-8, 0.1, 3
    ref_p, ref_m, ref_v = param.clone(), m.clone(), v.clone()
    reference_adamw(ref_p, expect, ref_m, ref_v, lr=lr, beta1=b1, beta2=b2, eps=eps, weight_decay=wd, step=step)
    # pads[p] is rank p's signal pad; slot (block, sender) = block * world + sender.  Pre-set the
    # peer's arrival in this rank's pad for every block the kernel may launch.
    pads = torch.zeros(world, 2 * _BLOCKS * world, dtype=torch.int32, device=dev)
    pads[rank, (1 - rank)::world] = 1
    shard16 = torch.empty(shard, device=dev, dtype=torch.bfloat16)
    grad_out = torch.full((shard,), float("nan"), device=dev)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    hyper = torch.tensor([lr, float(step), 1.0, 0.0], device=dev)
    ext.fsdp_reduce_scatter_adamw(staging[rank], [s.data_ptr() for s in staging], [pads[0].data_ptr(), pads[1].data_ptr()],
                                  rank, shard, valid, 1.0 / world, param, m, v, shard16, grad_out, hyper, b1, b2, eps, wd, 0,
                                  _BLOCKS, status, 0.1, -1)
    torch.cuda.synchronize()
    assert status[:2].tolist() == [1, 12], status.tolist()  # only the closing barrier (no live peer) ran out
    scale = float(expect.abs().max())
    assert float((grad_out - expect).abs().max()) <= 2e-6 * scale
    assert float((param - ref_p).abs().max()) < 2e-6
    assert float((m - ref_m).abs().max()) < 2e-6 and float((v - ref_v).abs().max()) < 2e-6
    assert torch.equal(shard16, param.bfloat16())


@pytest.mark.parametrize("rank", [0, 3])
def test_hybrid_shard_reduction_sums_every_replica_of_the_slice(rank: int) -> None:
    """Hybrid sharding: 2 replicas x 2 shards.  The kernel runs as rank ``rank`` of the 4-rank
    data-parallel x shard group and reduces slice ``rank % 2`` (its shard index) of all four ranks'
    staging buffers, which equals the reduce-scatter over the shard group followed by the
    all-reduce over the replicas."""
    ext = _ext()
    dev = torch.device("cuda")
    world, shards, shard = 4, 2, 65_536
    slice_index = rank % shards
    gen = torch.Generator(device="cuda").manual_seed(11 + rank)
    staging = [torch.randn(shards * shard, device=dev, generator=gen).bfloat16() for _ in range(world)]
    lo, hi = slice_index * shard, (slice_index + 1) * shard
    expect = sum(st[lo:hi].float() for st in staging) / world
    param = torch.randn(shard, device=dev, generator=gen)
    m, v = torch.zeros(shard, device=dev), torch.zeros(shard, device=dev)
    lr, b1, b2, eps, wd, step = 1e-3, 0.9, 0.95, 1e-8, 0.0, 1
    ref_p, ref_m, ref_v = param.clone(), m.clone(), v.clone()
    reference_adamw(ref_p, expect, ref_m, ref_v, lr=lr, beta1=b1, beta2=b2, eps=eps, weight_decay=wd, step=step)
    pads = torch.zeros(world, 2 * _BLOCKS * world, dtype=torch.int32, device=dev)
    for sender in range(world):
        if sender != rank:
            pads[rank, sender::world] = 1  # every peer's arrival at the opening barrier
    shard16 = torch.empty(shard, device=dev, dtype=torch.bfloat16)
    grad_out = torch.full((shard,), float("nan"), device=dev)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    hyper = torch.tensor([lr, float(step), 1.0, 0.0], device=dev)
    ext.fsdp_reduce_scatter_adamw(staging[rank], [t.data_ptr() for t in staging], [pads[q].data_ptr() for q in range(world)],
                                  rank, shard, shard, 1.0 / world, param, m, v, shard16, grad_out, hyper, b1, b2, eps, wd, 0,
                                  _BLOCKS, status, 0.1, slice_index)
    torch.cuda.synchronize()
    assert status[:2].tolist() == [1, 12], status.tolist()  # only the closing barrier (no live peers) ran out
    assert float((grad_out - expect).abs().max()) <= 2e-6 * float(expect.abs().max())
    assert float((param - ref_p).abs().max()) < 2e-6
    assert torch.equal(shard16, param.bfloat16())


@pytest.mark.parametrize("shard", [1_000_008, 12_345])
@pytest.mark.parametrize("copy_engine", [False, True])
def test_shard_all_gather(shard: int, copy_engine: bool) -> None:
    ext = _ext()
    dev = torch.device("cuda")
    shards = [torch.randn(shard, device=dev).bfloat16() for _ in range(2)]
    for rank in (0, 1):
        out = torch.full((2 * shard,), float("nan"), device=dev, dtype=torch.bfloat16)
        fn = ext.fsdp_all_gather_copy_engine if copy_engine else ext.fsdp_all_gather
        fn([s.data_ptr() for s in shards], out, shard, rank)
        torch.cuda.synchronize()
        assert torch.equal(out, torch.cat(shards))
