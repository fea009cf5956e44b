"""Failure detection on the GPU without a fault: a bounded wait that runs out reports through a status word.

The in-kernel collectives wait for their peers at per-block barriers.  Here one block runs that
barrier as rank 0 of a group of two whose "peer" signal pad is ordinary local memory that nothing
writes: the wait must give up after its deadline, record the stage in the status word and return,
leaving the context usable.  With the slot pre-set (the peer had already arrived) the same barrier
completes at once.  No kernel traps, faults or waits without a limit.
"""

from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ext():
    import hybrid_training.ops as ops

    return ops.extension()  # fails loudly when the native module is missing


def test_barrier_wait_runs_out_and_reports_its_stage() -> None:
    ext = _ext()
    pads = torch.zeros(2, 8, dtype=torch.int32, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ext.barrier_probe(pads, status, 0.25)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert status[:2].tolist() == [1, 99]
    assert 0.2 <= waited < 5.0, waited
    assert int(pads[1, 0]) == 1  # this rank still announced its arrival to the silent peer
    # The context is still usable after the timed-out wait.
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2


def test_barrier_completes_when_the_peer_has_arrived() -> None:
    ext = _ext()
    pads = torch.zeros(2, 8, dtype=torch.int32, device="cuda")
    pads[0, 1] = 1  # the peer's arrival flag in this rank's pad
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    ext.barrier_probe(pads, status, 2.0)
    torch.cuda.synchronize()
    assert status.tolist() == [0, 0, 0, 0]
    assert int(pads[0, 1]) == 0 and int(pads[1, 0]) == 1  # flag consumed; own arrival posted


def test_timed_out_wait_in_a_replayed_graph_raises_at_the_step_read() -> None:
    """A bounded wait that runs out inside a captured step surfaces when the engine reads the loss."""
    from types import SimpleNamespace

    from hybrid_training.distributed.symmetric import SymmetricWorkspace
    from hybrid_training.errors import KernelError
    from hybrid_training.training.engine import TrainingEngine

    ext = _ext()
    ws = SymmetricWorkspace.__new__(SymmetricWorkspace)  # status word only: no peer memory is needed here
    ws.status = torch.zeros(4, dtype=torch.int32, device="cuda")
    ws.group = SimpleNamespace(global_rank=0)
    engine = SimpleNamespace(context=SimpleNamespace(device=torch.device("cuda"), symmetric_workspaces=lambda: [ws]))
    pads = torch.zeros(2, 8, dtype=torch.int32, device="cuda")
    loss = torch.zeros(1, device="cuda")
    graph, side = torch.cuda.CUDAGraph(), torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
        loss.fill_(2.5)
        ext.barrier_probe(pads, ws.status, 0.1)  # the "peer" never arrives during a replay
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    assert ws.status.tolist() == [0, 0, 0, 0]  # capture recorded the kernel without running it
    graph.replay()
    with pytest.raises(KernelError, match="stage 99"):
        TrainingEngine.read_step_results(engine, loss, None)
    # The status word was cleared by the report; a clean step reads normally.
    assert ws.status.tolist() == [0, 0, 0, 0]
    loss.fill_(1.25)
    assert TrainingEngine.read_step_results(engine, loss, torch.full((1,), 3.0, device="cuda")) == (1.25, 3.0)
    del graph
