"""Multi-GPU paths on real devices: the in-kernel NVLink bucket all-reduce and DDP training over NCCL.

Each test spawns one process per GPU (two ranks) with the NCCL backend.  No rank is made to fail:
fault handling is covered by the CPU (Gloo) tests.
"""

from __future__ import annotations

import pytest
import torch

from hybrid_training.distributed import launch_workers

from . import dist_workers as W

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def test_native_all_gather_context_parallel_attention_matches_the_whole_sequence() -> None:
    results = launch_workers(W.gathered_attention_worker, 2, timeout_seconds=300, extra_env={"NCCL_NVLS_ENABLE": "0"})
    for r in results:
        v = r.value
        assert v["out"] < 1e-2 and v["dq"] < 1e-2 and v["dkv"] < 2e-2, v


def test_in_kernel_bucket_all_reduce_matches_nccl() -> None:
    results = launch_workers(W.bucket_allreduce_worker, 2, timeout_seconds=300,
                             extra_env={"NCCL_NVLS_ENABLE": "0"})
    for r in results:
        for err in r.value["errors"]:
            assert err < 1e-5, r.value["errors"]


def test_in_kernel_bucket_all_reduce_through_the_switch_matches_nccl() -> None:
    """The NVLS variant: the NVLink switch sums the copies (multimem.ld_reduce) and stores to all ranks."""
    results = launch_workers(W.bucket_allreduce_worker, 2, args=(True,), timeout_seconds=300,
                             extra_env={"NCCL_NVLS_ENABLE": "0"})
    if not results[0].value["nvls"]:
        pytest.skip("the NVLink switch offers no multicast address on this machine")
    for r in results:
        for err in r.value["errors"]:
            assert err < 1e-5, r.value["errors"]


def test_ddp_fused_and_nccl_reductions_train_alike() -> None:
    fused = launch_workers(W.ddp_cuda_worker, 2, args=(True, 3), timeout_seconds=300, extra_env={"NCCL_NVLS_ENABLE": "0"})
    nccl = launch_workers(W.ddp_cuda_worker, 2, args=(False, 3, True), timeout_seconds=300,
                          extra_env={"NCCL_NVLS_ENABLE": "0"})  # NCCL reduction with the per-bucket update
    assert fused[0].value["fused"] and not nccl[0].value["fused"]
    # DDP keeps every replica identical.
    for name, t in fused[0].value["full"].items():
        assert torch.equal(t, fused[1].value["full"][name]), name
    for a, b in zip(fused[0].value["losses"], nccl[0].value["losses"]):
        assert abs(a - b) < 1e-2 * max(1.0, abs(b)), (fused[0].value["losses"], nccl[0].value["losses"])


def test_ddp_optimizer_update_overlapped_with_the_backward_matches_the_step_after_it() -> None:
    """AdamW per bucket on the communication stream, eager and replayed from a CUDA graph."""
    base = launch_workers(W.ddp_cuda_worker, 2, args=(True, 4, False, False), timeout_seconds=300,
                          extra_env={"NCCL_NVLS_ENABLE": "0"})
    for graph in (False, True):
        over = launch_workers(W.ddp_cuda_worker, 2, args=(True, 4, True, graph), timeout_seconds=300,
                              extra_env={"NCCL_NVLS_ENABLE": "0"})
        for name, t in over[0].value["full"].items():
            assert torch.equal(t, over[1].value["full"][name]), name  # replicas stay identical
            ref = base[0].value["full"][name]
            assert torch.allclose(t, ref, atol=2e-3, rtol=2e-3), (name, float((t - ref).abs().max()))
        for a, b in zip(over[0].value["losses"], base[0].value["losses"]):
            assert abs(a - b) < 1e-2 * max(1.0, abs(b)), (over[0].value["losses"], base[0].value["losses"])


@pytest.mark.parametrize("sp", [True, False])
def test_fused_tensor_parallel_collectives_match_nccl_path(sp: bool) -> None:
    """SP: all-gather fused into the column GEMM's loads, reduce-scatter fused into the row GEMM's epilogue.
    No SP: the row output and the column input gradient summed by the in-kernel all-reduce."""
    results = launch_workers(W.tp_fused_collectives_worker, 2, args=(sp,), timeout_seconds=300,
                             extra_env={"NCCL_NVLS_ENABLE": "0"})
    for r in results:
        assert r.value["error_word"] == 0
        for key, err in r.value["errors"].items():
            assert err < 2e-2, (key, r.value["errors"])


def test_fsdp_llama_trains_on_two_gpus() -> None:
    results = launch_workers(W.llama_cuda_worker, 2, args=({"shard_parallel_size": 2}, True, 3), timeout_seconds=300,
                             extra_env={"NCCL_NVLS_ENABLE": "0"})
    losses = results[0].value["losses"]
    assert len(losses) == 3 and all(l == l and 0 < l < 20 for l in losses), losses
    assert losses == results[1].value["losses"]


def test_tensor_sequence_parallel_llama_fused_matches_nccl_path() -> None:
    topo = {"tensor_parallel_size": 2, "sequence_parallel_mode": "tensor_group"}
    fused = launch_workers(W.llama_cuda_worker, 2, args=(topo, True, 3), timeout_seconds=300, extra_env={"NCCL_NVLS_ENABLE": "0"})
    nccl = launch_workers(W.llama_cuda_worker, 2, args=(topo, False, 3), timeout_seconds=300, extra_env={"NCCL_NVLS_ENABLE": "0"})
    for a, b in zip(fused[0].value["losses"], nccl[0].value["losses"]):
        assert abs(a - b) < 2e-2 * max(1.0, abs(b)), (fused[0].value["losses"], nccl[0].value["losses"])


def test_fsdp_fused_reduce_scatter_adamw_and_all_gather_kernels() -> None:
    """One kernel: reduce-scatter over peer memory + cast + AdamW on the shard; P2P shard all-gather."""
    results = launch_workers(W.fsdp_fused_kernels_worker, 2, timeout_seconds=300, extra_env={"NCCL_NVLS_ENABLE": "0"})
    for r in results:
        for key, err in r.value["errors"].items():
            limit = 2e-6 if key.startswith(("grad", "param", "exp_avg")) else 0.0
            assert err <= limit, (key, r.value["errors"])


@pytest.mark.parametrize("accumulation", [1, 2])
def test_fsdp_fused_update_trains_like_nccl_path(accumulation: int) -> None:
    fused = launch_workers(W.fsdp_fused_update_worker, 2, args=(True, 3, accumulation), timeout_seconds=300,
                           extra_env={"NCCL_NVLS_ENABLE": "0"})
    nccl = launch_workers(W.fsdp_fused_update_worker, 2, args=(False, 3, accumulation), timeout_seconds=300,
                          extra_env={"NCCL_NVLS_ENABLE": "0"})
    assert fused[0].value["fused"] and not nccl[0].value["fused"]
    for a, b in zip(fused[0].value["losses"], nccl[0].value["losses"]):
        assert abs(a - b) < 1e-2 * max(1.0, abs(b)), (fused[0].value["losses"], nccl[0].value["losses"])
    assert fused[0].value["losses"] == fused[1].value["losses"]
    for name, t in fused[0].value["full"].items():
        ref = nccl[0].value["full"][name]
        err = float((t - ref).abs().max())
        assert err < 5e-3 * max(1.0, float(ref.abs().max())), (name, err)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="hybrid sharding (2 replicas x 2 shards) needs 4 GPUs")
def test_hybrid_sharding_fused_update_trains_like_nccl_path() -> None:
    """HSDP: one kernel sums every replica's slice over the 4 ranks and updates the shard, against
    NCCL reduce-scatter + replica all-reduce + the separate optimizer step."""
    fused = launch_workers(W.fsdp_fused_update_worker, 4, args=(True, 3, 1, 2), timeout_seconds=300,
                           extra_env={"NCCL_NVLS_ENABLE": "0"})
    nccl = launch_workers(W.fsdp_fused_update_worker, 4, args=(False, 3, 1, 2), timeout_seconds=300,
                          extra_env={"NCCL_NVLS_ENABLE": "0"})
    assert all(r.value["fused"] for r in fused) and not nccl[0].value["fused"]
    for a, b in zip(fused[0].value["losses"], nccl[0].value["losses"]):
        assert abs(a - b) < 1e-2 * max(1.0, abs(b)), (fused[0].value["losses"], nccl[0].value["losses"])
    for r in fused[1:]:
        assert r.value["losses"] == fused[0].value["losses"]
    for name, t in fused[0].value["full"].items():
        ref = nccl[0].value["full"][name]
        err = float((t - ref).abs().max())
        assert err < 5e-3 * max(1.0, float(ref.abs().max())), (name, err)
    # the replicas of a shard hold bitwise-identical parameters
    for name, t in fused[0].value["full"].items():
        assert torch.equal(t, fused[2].value["full"][name]), name
