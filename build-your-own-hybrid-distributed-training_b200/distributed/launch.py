"""Multi-process launcher for tests, benchmarks and examples.

``launch_workers(entrypoint, world_size, ...)`` spawns one child per rank with a
private rendezvous on ``127.0.0.1``, runs ``entrypoint(rank, world_size, *args,
**kwargs)`` in each, and returns one :class:`WorkerResult` per rank.  A failing
rank's traceback travels back as text; ranks that produce nothing before the
deadline are terminated and reported with the machine's load and memory, which
tells a real collective mismatch apart from an overloaded box.  API and
behaviour follow ``src/hybrid_training/distributed/launch.py:51-469``.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import pickle
import queue
import sys
import time
import traceback
from collections.abc import Callable, Sequence
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

from ..errors import DistributedInitializationError, format_error
from ..logging import configure_logging, get_logger
from .context import find_free_port

__all__ = ["WorkerFailure", "WorkerResult", "launch_workers", "torchrun_environment_summary"]

_LOG = get_logger(__name__)


@dataclass
class WorkerResult:
    rank: int
    value: Any = None
    traceback_text: str | None = None
    exit_code: int | None = None
    duration_seconds: float = 0.0

    @property
    def succeeded(self) -> bool:
        return self.traceback_text is None and self.exit_code in (0, None)


class WorkerFailure(DistributedInitializationError):
    """Raised when any rank fails or times out; carries every rank's result."""

    def __init__(self, message: str, results: Sequence[WorkerResult]) -> None:
        self.results = tuple(results)
        self.summary = message
        super().__init__(self._render(message))

    def _render(self, headline: str) -> str:
        out = [headline]
        for r in sorted(self.results, key=lambda r: r.rank):
            out.append(f"--- rank {r.rank}: {'ok' if r.succeeded else 'FAILED'} (exit_code={r.exit_code}, "
                       f"{r.duration_seconds:.2f}s) ---")
            if r.traceback_text:
                out.append(r.traceback_text.rstrip())
        return "\n".join(out)

    def detailed_report(self) -> str:
        return str(self)

    def failing_ranks(self) -> tuple[int, ...]:
        return tuple(r.rank for r in self.results if not r.succeeded)


@dataclass
class _Spec:
    rank: int
    world_size: int
    master_addr: str
    master_port: int
    entrypoint: Callable[..., Any]
    args: tuple[Any, ...]
    kwargs: dict[str, Any]
    extra_env: dict[str, str] = field(default_factory=dict)
    log_level: str = "WARNING"


def _child(spec: _Spec, results: Any) -> None:
    start = time.perf_counter()
    os.environ.update({
        "RANK": str(spec.rank), "WORLD_SIZE": str(spec.world_size), "LOCAL_RANK": str(spec.rank),
        "LOCAL_WORLD_SIZE": str(spec.world_size), "MASTER_ADDR": spec.master_addr, "MASTER_PORT": str(spec.master_port),
    })
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    os.environ.update(spec.extra_env)
    configure_logging(spec.log_level, force=True)
    code = 0
    try:
        import torch

        torch.set_num_threads(1)
        value = spec.entrypoint(spec.rank, spec.world_size, *spec.args, **spec.kwargs)
        result = WorkerResult(spec.rank, value, duration_seconds=time.perf_counter() - start)
    except BaseException:
        result = WorkerResult(spec.rank, None, traceback.format_exc(), duration_seconds=time.perf_counter() - start)
        code = 1
    try:
        blob = pickle.dumps(result, protocol=pickle.HIGHEST_PROTOCOL)
    except Exception:
        blob = pickle.dumps(WorkerResult(spec.rank, None, "the worker's return value could not be pickled:\n"
                                         + traceback.format_exc(), duration_seconds=time.perf_counter() - start))
        code = 1
    results.put(blob)
    sys.stdout.flush()
    sys.stderr.flush()
    sys.exit(code)


def _machine_state() -> str:
    parts = []
    try:
        l1, l5, _ = os.getloadavg()
        parts.append(f"load {l1:.1f}/{l5:.1f} over {os.cpu_count() or 1} core(s)")
    except OSError:
        pass
    try:
        info = {}
        for line in Path("/proc/meminfo").read_text().splitlines():
            key, _, rest = line.partition(":")
            if key in ("MemAvailable", "SwapTotal", "SwapFree"):
                info[key] = int(rest.split()[0]) * 1024
        if "MemAvailable" in info:
            swapped = info.get("SwapTotal", 0) - info.get("SwapFree", 0)
            parts.append(f"{info['MemAvailable'] >> 20} MiB available, {swapped >> 20} MiB swapped")
    except OSError:
        pass
    return ("  Machine at failure: " + "; ".join(parts) + ".") if parts else "  (machine state unavailable)"


def _require_picklable(obj: Any, what: str) -> None:
    try:
        pickle.dumps(obj)
    except Exception as exc:
        raise DistributedInitializationError(format_error(
            "launch.launch_workers", f"{what} is not picklable, and spawned workers receive their arguments by pickling",
            expected="a function defined at module level, with picklable arguments", observed=repr(obj)[:200],
            resolution="move the entrypoint to module scope and pass only picklable arguments")) from exc


_NO_RESULT = ("rank produced no result: it was still running at the deadline, or died before reporting.\n"
              "  1. a collective mismatch blocks a rank inside a collective its peers never issued;\n"
              "  2. an overloaded machine makes every rank slow (each spawned rank imports torch).\n")


def launch_workers(
    entrypoint: Callable[..., Any],
    world_size: int,
    *,
    args: Sequence[Any] = (),
    kwargs: dict[str, Any] | None = None,
    timeout_seconds: float = 180.0,
    start_method: str = "spawn",
    master_addr: str = "127.0.0.1",
    master_port: int | None = None,
    extra_env: dict[str, str] | None = None,
    log_level: str = "WARNING",
    raise_on_failure: bool = True,
) -> list[WorkerResult]:
    """Run ``entrypoint`` on ``world_size`` spawned ranks and gather their results."""
    if world_size < 1:
        raise DistributedInitializationError(format_error("launch.launch_workers", "at least one worker is needed",
                                                          expected=">= 1", observed=world_size, resolution="ask for one or more workers"))
    kwargs = dict(kwargs or {})
    if start_method == "spawn":
        _require_picklable(entrypoint, "the entrypoint")
        _require_picklable((tuple(args), kwargs), "the worker function and its arguments")
    port = master_port if master_port is not None else find_free_port(master_addr)
    ctx: Any = mp.get_context(start_method)
    inbox: Any = ctx.Queue()
    procs = []
    for rank in range(world_size):
        spec = _Spec(rank, world_size, master_addr, port, entrypoint, tuple(args), kwargs, dict(extra_env or {}), log_level)
        proc = ctx.Process(target=_child, args=(spec, inbox), daemon=False)
        proc.start()
        procs.append(proc)
    got: dict[int, WorkerResult] = {}
    deadline = time.monotonic() + timeout_seconds
    timed_out = False
    try:
        while len(got) < world_size:
            left = deadline - time.monotonic()
            if left <= 0:
                timed_out = True
                break
            try:
                item: WorkerResult = pickle.loads(inbox.get(timeout=min(left, 1.0)))
            except queue.Empty:
                if all(not p.is_alive() for p in procs) and inbox.empty():
                    break
                continue
            got[item.rank] = item
        for proc in procs:
            proc.join(timeout=0.0 if timed_out else max(deadline - time.monotonic(), 0.0))
            timed_out = timed_out or proc.is_alive()
    finally:
        for proc in procs:
            if proc.is_alive():
                proc.terminate()
        for proc in procs:
            proc.join(timeout=10.0)
            if proc.is_alive():
                proc.kill()
                proc.join(timeout=10.0)
        inbox.close()
    results = []
    for rank, proc in enumerate(procs):
        result = got.get(rank) or WorkerResult(rank, traceback_text=_NO_RESULT + _machine_state())
        result.exit_code = proc.exitcode
        results.append(result)
    failed = [r for r in results if not r.succeeded]
    if failed and raise_on_failure:
        raise WorkerFailure(format_error(
            "launch.launch_workers", f"{len(failed)} of {world_size} worker(s) {'timed out' if timed_out else 'failed'}",
            expected="all workers to finish and exit with status 0", observed=f"failing ranks: {[r.rank for r in failed]}",
            resolution="see each failing rank's traceback below; a rank without one was still waiting inside a collective"), results)
    return results


def torchrun_environment_summary(env: dict[str, str] | None = None) -> dict[str, str]:
    source = os.environ if env is None else env
    names = ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT", "GROUP_RANK",
             "ROLE_RANK", "TORCHELASTIC_RUN_ID", "CUDA_VISIBLE_DEVICES", "OMP_NUM_THREADS", "NCCL_DEBUG")
    return {n: source.get(n, "<unset>") for n in names}
