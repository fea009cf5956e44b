"""Checkpoint format, integrity checks, resume and resharding across world sizes (CPU/Gloo)."""

from __future__ import annotations

import json
import shutil
from pathlib import Path

import pytest
import torch

from hybrid_training.checkpoint import (
    CheckpointManifest,
    ShardRecord,
    TensorRecord,
    checkpoint_directory_name,
    find_latest_checkpoint,
    inspect_checkpoint,
    prune_checkpoints,
    shard_filename,
    validate_shard_filename,
)
from hybrid_training.checkpoint.format import resolve_inside, staging_directory_name
from hybrid_training.distributed import launch_workers
from hybrid_training.errors import CheckpointCorruptionError, CheckpointError, IncompleteCheckpointError

from . import dist_workers as W


def test_names_and_path_safety(tmp_path: Path) -> None:
    assert checkpoint_directory_name(7) == "checkpoint-step-000007"
    assert shard_filename(3) == "rank-00003.pt"
    assert staging_directory_name("checkpoint-step-000007", "abc").startswith(".staging-checkpoint-step-000007-")
    for bad in ("../etc/passwd", "rank-1.pt", "x.pt"):
        with pytest.raises(CheckpointError):
            validate_shard_filename(bad)
    (tmp_path / "out").mkdir()
    with pytest.raises(CheckpointError):
        resolve_inside(tmp_path / "out", "../escape")


def _record(key: str, numel: int, shards: list[tuple[int, int]]) -> TensorRecord:
    r = TensorRecord(key=key, name=key, global_shape=(numel,), dtype="torch.float32")
    for i, (off, n) in enumerate(shards):
        r.shards.append(ShardRecord(rank=i, file=shard_filename(i), offset=off, length=n, key=f"model::{key}@{off}"))
    return r


def test_manifest_validation() -> None:
    _record("a", 10, [(0, 5), (5, 5)]).validate()
    with pytest.raises(CheckpointCorruptionError):
        _record("a", 10, [(0, 6), (5, 5)]).validate()
    with pytest.raises(IncompleteCheckpointError):
        _record("a", 10, [(0, 4), (5, 5)]).validate()
    m = CheckpointManifest()
    m.tensors["a"] = _record("a", 10, [(0, 10)])
    with pytest.raises(IncompleteCheckpointError):
        m.validate()  # not marked complete
    m.complete = True
    with pytest.raises(IncompleteCheckpointError):
        m.validate()  # no integrity record for the file
    assert CheckpointManifest.from_dict(json.loads(m.to_json())).tensors["a"].numel == 10


def _cfg(world: int, shard: int, dp: int = 1, tp: int = 1, steps: int = 4) -> dict:
    return {"backend": "gloo", "device": "cpu",
            "topology": {"shard_parallel_size": shard, "data_parallel_size": dp, "tensor_parallel_size": tp},
            "model": {"kind": "transformer", "hidden_size": 32, "num_layers": 2, "num_heads": 4, "vocab_size": 64,
                      "max_sequence_length": 16},
            "data": {"micro_batch_size": 8 // (world // tp), "sequence_length": 16, "num_train_samples": 256,
                     "num_eval_samples": 0, "shuffle": False},
            "optimizer": {"learning_rate": 0.003}, "fsdp": {"auto_wrap_min_num_params": 1000},
            "training": {"max_steps": steps, "log_every_steps": 0}}


@pytest.mark.distributed
def test_save_fsdp4_reload_fsdp2_and_ddp2_bitwise(tmp_path: Path) -> None:
    saved = launch_workers(W.engine_worker, 4, args=(_cfg(4, 4), 3, str(tmp_path), None), timeout_seconds=600)
    path = saved[0].value["path"]
    assert path and Path(path, "manifest.json").is_file()
    full_before = saved[0].value["full"]
    info = inspect_checkpoint(path)
    assert info["complete"] and info["writer_world_size"] == 4 and info["verification"]["files_verified"] == 4
    for shard, dp in ((2, 1), (1, 2)):
        reloaded = launch_workers(W.engine_worker, 2, args=(_cfg(2, shard, dp), 3, None, path), timeout_seconds=600)
        for name, t in full_before.items():
            assert torch.equal(reloaded[0].value["full"][name], t), (shard, dp, name)


@pytest.mark.distributed
def test_resume_reproduces_uninterrupted_run(tmp_path: Path) -> None:
    straight = launch_workers(W.engine_worker, 2, args=(_cfg(2, 2), 4, None, None), timeout_seconds=600)
    first = launch_workers(W.engine_worker, 2, args=(_cfg(2, 2), 2, str(tmp_path), None), timeout_seconds=600)
    resumed = launch_workers(W.engine_worker, 2, args=(_cfg(2, 2), 4, None, first[0].value["path"]), timeout_seconds=600)
    assert resumed[0].value["losses"] == straight[0].value["losses"][2:]
    for name, t in straight[0].value["full"].items():
        assert torch.equal(resumed[0].value["full"][name], t), name


@pytest.mark.distributed
def test_hybrid_dp2_tp2_saves_and_restores_at_dp1_tp2_bitwise(tmp_path: Path) -> None:
    """The benchmark's reshard rule at small scale: DP2 x TP2 -> DP1 x TP2 (tensor width unchanged)."""
    saved = launch_workers(W.engine_worker, 4, args=(_cfg(4, 1, dp=2, tp=2), 2, str(tmp_path), None), timeout_seconds=600)
    restored = launch_workers(W.engine_worker, 2, args=(_cfg(2, 1, dp=1, tp=2), 2, None, saved[0].value["path"]),
                              timeout_seconds=600)
    for rank in range(2):
        for name, t in saved[rank].value["full"].items():
            assert torch.equal(restored[rank].value["full"][name], t), (rank, name)


@pytest.mark.distributed
def test_corruption_and_topology_errors_are_detected(tmp_path: Path) -> None:
    saved = launch_workers(W.engine_worker, 2, args=(_cfg(2, 2), 1, str(tmp_path / "c"), None), timeout_seconds=600)
    path = Path(saved[0].value["path"])

    def variant(name: str) -> Path:
        dst = tmp_path / name / path.name
        shutil.copytree(path, dst)
        return dst

    flipped = variant("flip")
    blob = bytearray((flipped / "rank-00001.pt").read_bytes())
    blob[-20] ^= 0xFF
    (flipped / "rank-00001.pt").write_bytes(bytes(blob))
    with pytest.raises(CheckpointCorruptionError):
        inspect_checkpoint(flipped)
    truncated = variant("trunc")
    data = (truncated / "rank-00000.pt").read_bytes()
    (truncated / "rank-00000.pt").write_bytes(data[:-10])
    with pytest.raises(CheckpointCorruptionError):
        inspect_checkpoint(truncated)
    missing = variant("missing")
    (missing / "rank-00001.pt").unlink()
    with pytest.raises(IncompleteCheckpointError):
        inspect_checkpoint(missing)
    nomanifest = variant("nomanifest")
    (nomanifest / "manifest.json").unlink()
    with pytest.raises(IncompleteCheckpointError):
        inspect_checkpoint(nomanifest)
    edited = variant("edited")
    m = json.loads((edited / "manifest.json").read_text())
    m["complete"] = False
    (edited / "manifest.json").write_text(json.dumps(m))
    with pytest.raises(IncompleteCheckpointError):
        inspect_checkpoint(edited)
    tp_cfg = _cfg(2, 1, tp=2)
    results = launch_workers(W.engine_worker, 2, args=(tp_cfg, 1, None, str(path)), timeout_seconds=600, raise_on_failure=False)
    assert all("CheckpointTopologyError" in (r.traceback_text or "") for r in results)


def test_prune_and_find_latest(tmp_path: Path) -> None:
    for step in (1, 5, 3):
        d = tmp_path / checkpoint_directory_name(step)
        d.mkdir()
        (d / "manifest.json").write_text("{}")
    (tmp_path / checkpoint_directory_name(9)).mkdir()  # unpublished: no manifest
    assert find_latest_checkpoint(tmp_path).name == checkpoint_directory_name(5)
    removed = prune_checkpoints(tmp_path, keep_last=2)
    assert sorted(p.name for p in removed) == [checkpoint_directory_name(1), checkpoint_directory_name(3)]


@pytest.fixture(scope="module")
def fsdp_checkpoint(tmp_path_factory: pytest.TempPathFactory) -> Path:
    root = tmp_path_factory.mktemp("integrity")
    saved = launch_workers(W.engine_worker, 2, args=(_cfg(2, 2), 1, str(root), None), timeout_seconds=600)
    return Path(saved[0].value["path"])


def _copy(src: Path, tmp_path: Path, name: str) -> Path:
    dst = tmp_path / name / src.name
    shutil.copytree(src, dst)
    return dst


def test_publish_protocol_leaves_manifest_last_and_no_staging(fsdp_checkpoint: Path) -> None:
    manifest_time = (fsdp_checkpoint / "manifest.json").stat().st_mtime_ns
    for f in fsdp_checkpoint.iterdir():
        assert f.stat().st_mtime_ns <= manifest_time, f"{f.name} written after the manifest"
    assert not [p for p in fsdp_checkpoint.parent.iterdir() if p.name.startswith(".staging-")]
    summary = inspect_checkpoint(fsdp_checkpoint)
    assert summary["complete"] and summary["verification"]["files_verified"] == 2


def test_version_mismatch_is_rejected(fsdp_checkpoint: Path, tmp_path: Path) -> None:
    from hybrid_training.errors import CheckpointVersionError

    bad = _copy(fsdp_checkpoint, tmp_path, "version")
    m = json.loads((bad / "manifest.json").read_text())
    m["format_version"] = "9.0"
    (bad / "manifest.json").write_text(json.dumps(m))
    with pytest.raises(CheckpointVersionError):
        inspect_checkpoint(bad)


def test_dropped_shard_record_breaks_coverage(fsdp_checkpoint: Path, tmp_path: Path) -> None:
    bad = _copy(fsdp_checkpoint, tmp_path, "dropped")
    m = json.loads((bad / "manifest.json").read_text())
    key = next(k for k, r in m["tensors"].items() if len(r["shards"]) == 2)
    m["tensors"][key]["shards"].pop()
    (bad / "manifest.json").write_text(json.dumps(m))
    with pytest.raises(CheckpointError):
        inspect_checkpoint(bad)


def test_hostile_file_name_in_manifest_is_rejected(fsdp_checkpoint: Path, tmp_path: Path) -> None:
    bad = _copy(fsdp_checkpoint, tmp_path, "hostile")
    m = json.loads((bad / "manifest.json").read_text())
    key = next(iter(m["tensors"]))
    m["tensors"][key]["shards"][0]["file"] = "../../outside.pt"
    (bad / "manifest.json").write_text(json.dumps(m))
    with pytest.raises(CheckpointError):
        inspect_checkpoint(bad)


def test_corruption_is_caught_by_a_real_load(fsdp_checkpoint: Path, tmp_path: Path) -> None:
    bad = _copy(fsdp_checkpoint, tmp_path, "load")
    blob = bytearray((bad / "rank-00000.pt").read_bytes())
    blob[len(blob) // 2] ^= 0x5A
    (bad / "rank-00000.pt").write_bytes(bytes(blob))
    results = launch_workers(W.engine_worker, 2, args=(_cfg(2, 2), 0, None, str(bad)), timeout_seconds=600,
                             raise_on_failure=False)
    assert all("CheckpointCorruptionError" in (r.traceback_text or "") for r in results)


def test_verify_files_returns_the_recorded_digests(fsdp_checkpoint: Path) -> None:
    from hybrid_training.checkpoint.reshard import verify_files

    manifest = CheckpointManifest.read(fsdp_checkpoint / "manifest.json")
    digests = verify_files(fsdp_checkpoint, manifest)
    assert set(digests) == {"rank-00000.pt", "rank-00001.pt"}
    assert all(digests[name] == record.sha256 for name, record in manifest.files.items())


def test_metadata_is_plain_json_with_the_training_state(fsdp_checkpoint: Path) -> None:
    from hybrid_training.checkpoint import read_metadata

    meta = read_metadata(fsdp_checkpoint)
    json.dumps(meta, allow_nan=False)  # no tensors, no NaN
    assert meta["training_state"]["step"] == 1 and meta["world_size"] == 2
    assert meta["rng"]["saved"] and meta["rng"]["ranks"] == [0, 1]


def test_manifest_describes_global_tensors_split_in_flat_intervals(fsdp_checkpoint: Path) -> None:
    manifest = CheckpointManifest.read(fsdp_checkpoint / "manifest.json")
    model = {k: r for k, r in manifest.tensors.items() if r.category == "model"}
    assert model and all(r.covered_elements() == r.numel for r in model.values())
    # full-shard over 2 ranks: some tensor is split between the two payload files
    assert any(len({s.file for s in r.shards}) == 2 for r in model.values())
    optimizer = {k: r for k, r in manifest.tensors.items() if r.category == "optimizer"}
    assert {r.state_name for r in optimizer.values()} == {"exp_avg", "exp_avg_sq"}


def test_swapped_payload_files_fail_verification(fsdp_checkpoint: Path, tmp_path: Path) -> None:
    bad = _copy(fsdp_checkpoint, tmp_path, "swapped")
    a, b = (bad / "rank-00000.pt").read_bytes(), (bad / "rank-00001.pt").read_bytes()
    (bad / "rank-00000.pt").write_bytes(b)
    (bad / "rank-00001.pt").write_bytes(a)
    with pytest.raises(CheckpointCorruptionError):
        inspect_checkpoint(bad)


def test_a_link_that_leaves_the_directory_is_rejected(fsdp_checkpoint: Path, tmp_path: Path) -> None:
    bad = _copy(fsdp_checkpoint, tmp_path, "symlink")
    outside = tmp_path / "elsewhere.pt"
    outside.write_bytes((bad / "rank-00001.pt").read_bytes())
    (bad / "rank-00001.pt").unlink()
    (bad / "rank-00001.pt").symlink_to(outside)
    with pytest.raises(CheckpointError):
        inspect_checkpoint(bad)


def test_saving_twice_at_one_step_fails_on_every_rank(tmp_path: Path) -> None:
    root = tmp_path / "twice"
    launch_workers(W.engine_worker, 2, args=(_cfg(2, 2), 1, str(root), None), timeout_seconds=600)
    again = launch_workers(W.engine_worker, 2, args=(_cfg(2, 2), 1, str(root), None), timeout_seconds=600,
                           raise_on_failure=False)
    for r in again:
        assert "CheckpointError" in (r.traceback_text or "") and "reserve" in (r.traceback_text or ""), r.traceback_text
    assert len([p for p in root.iterdir() if p.name.startswith("checkpoint-step-")]) == 1
    assert not [p for p in root.iterdir() if p.name.startswith(".staging-")]


def test_a_rank_that_cannot_write_makes_every_rank_fail(tmp_path: Path) -> None:
    """A write failure on one rank (not the coordinator) is voted on: all ranks raise, nothing is published."""
    results = launch_workers(W.checkpoint_write_failure_worker, 2, args=(str(tmp_path / "voted"),), timeout_seconds=600,
                             raise_on_failure=False)
    for r in results:
        assert r.value is not None and r.value["raised"], r.traceback_text
        assert "rank 1" in r.value["message"] and "write" in r.value["message"]
    assert not [p for p in (tmp_path / "voted").iterdir() if p.name.startswith("checkpoint-step-")]
