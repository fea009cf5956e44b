"""Distributed context: launch environment, backend/device choice, process groups.

``init_distributed`` accepts the same arguments as the reference
(``src/hybrid_training/distributed/context.py:565-747``): it reads the torchrun
environment (or explicit ``rank``/``world_size``, or falls back to a one-rank
group on a free port), resolves ``auto`` to NCCL when every local rank has its
own GPU, **sets the CUDA device before NCCL initialisation**, creates the
default group with a timeout, builds the grid and the registry, and installs
the rank tag for logging.  A second active context in one process is refused.
"""

from __future__ import annotations

import os
import socket
from collections.abc import Iterator
from contextlib import contextmanager
from dataclasses import dataclass
from datetime import timedelta
from typing import Any

import torch
import torch.distributed as dist

from ..config import ExperimentConfig, TopologyConfig
from ..errors import DistributedInitializationError, format_error
from ..logging import LogContext, get_logger, set_log_context
from .groups import GroupHandle, ProcessGroupRegistry
from .topology import ParallelTopology, RankCoordinates

__all__ = [
    "DistributedContext",
    "LaunchEnvironment",
    "current_context",
    "distributed_context",
    "find_free_port",
    "init_distributed",
    "is_context_active",
]

_LOG = get_logger(__name__)
_ACTIVE: DistributedContext | None = None
_TORCHRUN_VARS = ("RANK", "WORLD_SIZE")


def find_free_port(host: str = "127.0.0.1") -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sock:
        sock.bind((host, 0))
        return int(sock.getsockname()[1])


def _init_error(problem: str, fix: str, **kw: Any) -> DistributedInitializationError:
    op = kw.pop("op", "context")
    return DistributedInitializationError(format_error(op, problem, resolution=fix, **kw))


@dataclass(frozen=True)
class LaunchEnvironment:
    """Where this process sits in the job, as told by the launcher."""

    rank: int
    world_size: int
    local_rank: int
    local_world_size: int
    master_addr: str
    master_port: int

    def __post_init__(self) -> None:
        op = "context.LaunchEnvironment"
        if self.world_size < 1:
            raise _init_error("the world has at least one rank", "check WORLD_SIZE", op=op, rank=self.rank, expected=">= 1",
                              observed=self.world_size)
        if not 0 <= self.rank < self.world_size:
            raise _init_error("the rank is not below the world size", "check RANK", op=op, rank=self.rank, world_size=self.world_size,
                              expected=f"0 <= rank < {self.world_size}", observed=self.rank)
        if not 0 <= self.local_rank < max(self.local_world_size, 1):
            raise _init_error("the local rank is not below the node's process count", "look at the LOCAL_RANK and LOCAL_WORLD_SIZE the launcher exported", op=op, rank=self.rank,
                              world_size=self.world_size, expected=f"0 <= local_rank < {self.local_world_size}",
                              observed=self.local_rank)
        if not 1 <= self.master_port <= 65535:
            raise _init_error("MASTER_PORT is not a TCP port number", "check MASTER_PORT", op=op, rank=self.rank,
                              world_size=self.world_size, expected="1..65535", observed=self.master_port)

    @classmethod
    def from_environment(cls, env: dict[str, str] | None = None, *, allow_single_process: bool = True) -> LaunchEnvironment:
        source = dict(os.environ if env is None else env)
        op = "context.LaunchEnvironment.from_environment"
        present = [v for v in _TORCHRUN_VARS if v in source]
        if not present:
            if not allow_single_process:
                raise _init_error("the environment has no torchrun-style launch variables",
                                  "launch with torchrun, or pass rank/world_size to init_distributed()", op=op,
                                  expected="RANK, WORLD_SIZE to be set", observed="none set")
            port = find_free_port()
            _LOG.info("no torchrun environment; running single-process on port %d", port)
            return cls(0, 1, 0, 1, "127.0.0.1", port)
        if len(present) != len(_TORCHRUN_VARS):
            missing = [v for v in _TORCHRUN_VARS if v not in source]
            raise _init_error("the launch environment is only partially set", f"export what is missing: {missing}",
                              op=op, expected=list(_TORCHRUN_VARS), observed=present)

        def read(name: str, default: int | None = None) -> int:
            raw = source.get(name)
            if raw is None:
                if default is None:
                    raise _init_error(f"{name} has to be set by the launcher", f"export {name}", op=op)
                return default
            try:
                return int(raw)
            except ValueError as exc:
                raise _init_error(f"{name} is not an integer", f"export {name} written as a base-10 integer", op=op,
                                  expected="an integer", observed=raw) from exc

        rank, world = read("RANK"), read("WORLD_SIZE")
        return cls(rank, world, read("LOCAL_RANK", rank), read("LOCAL_WORLD_SIZE", world),
                   source.get("MASTER_ADDR", "127.0.0.1"), read("MASTER_PORT", 29500))


def _resolve_backend_and_device(backend: str, device: str, env: LaunchEnvironment) -> tuple[str, torch.device]:
    op = "context.resolve_backend"
    gpus = torch.cuda.device_count() if torch.cuda.is_available() else 0
    enough = gpus >= env.local_world_size
    if backend == "nccl" or device == "cuda":
        if gpus == 0:
            raise _init_error("NCCL on CUDA was asked for, but this process sees no GPU", "run on CPU with backend='gloo', device='cpu'",
                              op=op, rank=env.rank, world_size=env.world_size, expected=">= 1 CUDA device", observed=gpus)
        if backend == "nccl" and not enough:
            raise _init_error("NCCL needs one CUDA device per local process; sharing a device hangs instead of failing",
                              "lower --nproc-per-node to the GPU count, or use gloo on cpu", op=op, rank=env.rank,
                              world_size=env.world_size, expected=f">= {env.local_world_size} CUDA devices", observed=gpus)
        if backend == "nccl" and not dist.is_nccl_available():
            raise _init_error("the installed PyTorch was built without NCCL", "use a CUDA build of PyTorch", op=op, rank=env.rank)
        return ("nccl" if backend in ("auto", "nccl") else backend), torch.device("cuda", env.local_rank)
    if backend == "gloo" or device == "cpu":
        return "gloo", torch.device("cpu")
    if enough and gpus > 0 and dist.is_nccl_available():
        return "nccl", torch.device("cuda", env.local_rank)
    if gpus > 0:
        _LOG.warning("backend='auto': %d GPU(s) for %d local processes; falling back to gloo/cpu", gpus, env.local_world_size)
    return "gloo", torch.device("cpu")


class DistributedContext:
    """Owns the default process group (if it created it), the device and the registry."""

    def __init__(self, env: LaunchEnvironment, backend: str, device: torch.device, topology: ParallelTopology,
                 groups: ProcessGroupRegistry, *, owns_process_group: bool) -> None:
        self._env = env
        self._backend = backend
        self._device = device
        self._topology = topology
        self._groups = groups
        self._owns_pg = owns_process_group
        self._active = True
        self._symmetric: dict[str, Any] = {}

    rank = property(lambda self: self._env.rank)
    local_rank = property(lambda self: self._env.local_rank)
    world_size = property(lambda self: self._env.world_size)
    local_world_size = property(lambda self: self._env.local_world_size)
    backend = property(lambda self: self._backend)
    device = property(lambda self: self._device)
    env = property(lambda self: self._env)
    topology = property(lambda self: self._topology)
    groups = property(lambda self: self._groups)
    is_primary = property(lambda self: self._env.rank == 0)
    is_active = property(lambda self: self._active)

    @property
    def coordinates(self) -> RankCoordinates:
        return self._topology.coordinates_of(self._env.rank)

    def group(self, name: str) -> GroupHandle:
        return self._groups.get(name)

    def is_group_primary(self, name: str) -> bool:
        return self._groups.get(name).local_rank == 0

    def symmetric_workspace(self, group_name: str) -> Any:
        """Lazily created peer-mapped workspace for in-kernel collectives over ``group_name``.

        Returns ``None`` when the group is trivial, the job is not on CUDA, or
        peer memory cannot be established (the NCCL path is then used).
        """
        if group_name not in self._symmetric:
            from .symmetric import SymmetricWorkspace

            self._symmetric[group_name] = SymmetricWorkspace.create(self.group(group_name), self._device)
        return self._symmetric[group_name]

    def symmetric_workspaces(self) -> list[Any]:
        """Every peer-mapped workspace created so far (their status words report in-kernel timeouts)."""
        return [ws for ws in self._symmetric.values() if ws is not None]

    def barrier(self, group: str = "world", *, label: str = "") -> None:
        self._require_active("context.barrier")
        handle = self._groups.get(group)
        if handle.is_trivial:
            return
        _LOG.debug("barrier(%s)%s", group, f" [{label}]" if label else "")
        if self._backend == "nccl":
            dist.barrier(group=handle.process_group, device_ids=[self._device.index])
        else:
            dist.barrier(group=handle.process_group)

    def synchronize_device(self) -> None:
        if self._device.type == "cuda":
            torch.cuda.synchronize(self._device)

    def shutdown(self) -> None:
        """Release symmetric workspaces, sub-groups and (if owned) the default group."""
        global _ACTIVE
        if not self._active:
            return
        self._active = False
        try:
            for workspace in self._symmetric.values():
                if workspace is not None:
                    workspace.close()
            self._symmetric.clear()
            self._groups.destroy()
            if self._owns_pg and dist.is_initialized():
                dist.destroy_process_group()
        finally:
            if _ACTIVE is self:
                _ACTIVE = None
            set_log_context(LogContext())

    def __enter__(self) -> DistributedContext:
        return self

    def __exit__(self, *exc: object) -> None:
        self.shutdown()

    def _require_active(self, operation: str) -> None:
        if not self._active:
            raise _init_error("this context was already shut down", "call init_distributed() again for a fresh context",
                              op=operation, rank=self.rank, world_size=self.world_size)

    def describe(self) -> str:
        return (f"{self._topology.describe(self.rank)}\n  backend={self._backend} device={self._device} "
                f"local_rank={self.local_rank}/{self.local_world_size}")

    def __repr__(self) -> str:
        return f"DistributedContext(rank={self.rank}/{self.world_size}, backend={self._backend}, device={self._device}, {self._topology!r})"


def init_distributed(
    topology: TopologyConfig | ExperimentConfig | None = None,
    *,
    backend: str = "auto",
    device: str = "auto",
    timeout_seconds: float = 300.0,
    rank: int | None = None,
    world_size: int | None = None,
    local_rank: int | None = None,
    master_addr: str | None = None,
    master_port: int | None = None,
    env: dict[str, str] | None = None,
    allow_single_process: bool = True,
) -> DistributedContext:
    """Bring up the process group and the 4-D grid; see the module docstring."""
    global _ACTIVE
    if _ACTIVE is not None and _ACTIVE.is_active:
        raise _init_error("this process already has an active distributed context",
                          "call shutdown() on it first, or use distributed_context()", op="context.init_distributed",
                          rank=_ACTIVE.rank, world_size=_ACTIVE.world_size)
    if isinstance(topology, ExperimentConfig):
        topo_cfg: TopologyConfig | None = topology.topology
        backend, device, timeout_seconds = topology.backend, topology.device, topology.timeout_seconds
    else:
        topo_cfg = topology
    if rank is not None or world_size is not None:
        if rank is None or world_size is None:
            raise _init_error("an explicit rank needs an explicit world_size, and the other way round", "give both or leave both to the environment",
                              op="context.init_distributed", expected="both or neither",
                              observed=f"rank={rank}, world_size={world_size}")
        launch = LaunchEnvironment(rank, world_size, rank if local_rank is None else local_rank, world_size,
                                   master_addr or "127.0.0.1", master_port if master_port is not None else find_free_port())
    else:
        launch = LaunchEnvironment.from_environment(env, allow_single_process=allow_single_process)
        if master_addr is not None or master_port is not None:
            launch = LaunchEnvironment(launch.rank, launch.world_size, launch.local_rank, launch.local_world_size,
                                       master_addr or launch.master_addr,
                                       master_port if master_port is not None else launch.master_port)
    backend_name, dev = _resolve_backend_and_device(backend, device, launch)
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    preexisting = dist.is_initialized()
    if preexisting:
        if dist.get_world_size() != launch.world_size:
            raise _init_error("a process group of another size is already initialised",
                              "destroy the existing process group first", op="context.init_distributed",
                              rank=launch.rank, world_size=launch.world_size, expected=launch.world_size,
                              observed=dist.get_world_size())
    else:
        os.environ.setdefault("MASTER_ADDR", launch.master_addr)
        os.environ.setdefault("MASTER_PORT", str(launch.master_port))
        kwargs: dict[str, Any] = {}
        if dev.type == "cuda":
            kwargs["device_id"] = dev
        dist.init_process_group(backend=backend_name, init_method=f"tcp://{launch.master_addr}:{launch.master_port}",
                                rank=launch.rank, world_size=launch.world_size,
                                timeout=timedelta(seconds=timeout_seconds), **kwargs)
    try:
        topo_cfg = topo_cfg or TopologyConfig(data_parallel_size=launch.world_size)
        grid = ParallelTopology(topo_cfg, launch.world_size)
        registry = ProcessGroupRegistry(grid, launch.rank, timeout=timedelta(seconds=timeout_seconds))
    except Exception:
        if not preexisting and dist.is_initialized():
            dist.destroy_process_group()
        raise
    context = DistributedContext(launch, backend_name, dev, grid, registry, owns_process_group=not preexisting)
    _ACTIVE = context
    set_log_context(LogContext(launch.rank, launch.world_size, launch.local_rank, grid.coordinates_of(launch.rank).label()))
    _LOG.info("context up: %s on %s, grid %s", backend_name, dev, grid)
    return context


@contextmanager
def distributed_context(topology: TopologyConfig | ExperimentConfig | None = None, **kwargs: Any) -> Iterator[DistributedContext]:
    context = init_distributed(topology, **kwargs)
    try:
        yield context
    finally:
        context.shutdown()


def current_context() -> DistributedContext:
    if _ACTIVE is None or not _ACTIVE.is_active:
        raise _init_error("init_distributed() has not been called in this process (or the context was shut down)", "call init_distributed() first",
                          op="context.current_context")
    return _ACTIVE


def is_context_active() -> bool:
    return _ACTIVE is not None and _ACTIVE.is_active
