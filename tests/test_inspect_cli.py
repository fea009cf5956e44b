"""The checkpoint inspector CLI (``hybrid-inspect-checkpoint``) on a checkpoint written by 2 FSDP ranks.

Reference behaviour: ``scripts/inspect_checkpoint.py:65-185`` (summary, ``--json``, ``--tensors``,
``--plan``, ``--no-verify``; exit codes 0 valid / 1 invalid / 2 bad usage).
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest

from hybrid_training.checkpoint.reader import _console_main
from hybrid_training.distributed import launch_workers

from . import dist_workers as W

pytestmark = pytest.mark.distributed


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory: pytest.TempPathFactory) -> Path:
    root = tmp_path_factory.mktemp("ckpt")
    cfg = {"backend": "gloo", "device": "cpu", "topology": {"shard_parallel_size": 2},
           "model": {"kind": "transformer", "hidden_size": 32, "num_layers": 2, "num_heads": 4, "vocab_size": 64,
                     "max_sequence_length": 16},
           "data": {"micro_batch_size": 2, "sequence_length": 16, "num_train_samples": 64, "num_eval_samples": 0},
           "fsdp": {"auto_wrap_min_num_params": 1000}, "training": {"max_steps": 2, "log_every_steps": 0}}
    results = launch_workers(W.engine_worker, 2, args=(cfg, 2, str(root), None), timeout_seconds=300)
    return Path(results[0].value["path"])


def test_summary_and_json(checkpoint: Path, capsys: pytest.CaptureFixture[str]) -> None:
    assert _console_main([str(checkpoint)]) == 0
    text = capsys.readouterr().out
    assert "ranks that wrote it  2" in text and "files verified         2 / 2" in text
    assert _console_main([str(checkpoint), "--json"]) == 0
    summary = json.loads(capsys.readouterr().out)
    assert summary["writer_world_size"] == 2 and summary["verification"]["files_verified"] == 2
    assert summary["tensor_counts"]["model"] > 0 and summary["tensor_counts"]["optimizer"] > 0


def test_tensors_and_plans(checkpoint: Path, capsys: pytest.CaptureFixture[str]) -> None:
    assert _console_main([str(checkpoint), "--tensors", "--limit", "3", "--no-verify"]) == 0
    text = capsys.readouterr().out
    assert "tensors" in text and "more" in text and "not verified" in text
    manifest = json.loads((checkpoint / "manifest.json").read_text())
    key = next(k for k, r in manifest["tensors"].items() if r["category"] == "model" and len(r["shards"]) == 2)
    assert _console_main([str(checkpoint), "--plan", key, "--json"]) == 0
    plan = json.loads(capsys.readouterr().out)["plan"]
    assert {s["file"] for s in plan["sources"]} == {"rank-00000.pt", "rank-00001.pt"}
    assert _console_main([str(checkpoint), "--plan", key, "--reshard-to", "1", "--json"]) == 0
    one = json.loads(capsys.readouterr().out)["plan"]
    assert len(one) == 1 and one[0]["files"] == ["rank-00000.pt", "rank-00001.pt"]


def test_exit_codes(checkpoint: Path, tmp_path: Path, capsys: pytest.CaptureFixture[str]) -> None:
    assert _console_main([str(tmp_path / "missing")]) == 2
    assert _console_main([str(checkpoint), "--plan", "no.such.tensor"]) == 2
    broken = tmp_path / "broken"
    broken.mkdir()
    for f in checkpoint.iterdir():
        (broken / f.name).write_bytes(f.read_bytes())
    payload = broken / "rank-00001.pt"
    payload.write_bytes(payload.read_bytes()[:-7])
    assert _console_main([str(broken)]) == 1
    assert _console_main([str(broken), "--no-verify"]) == 0
    capsys.readouterr()
