"""Peer-mapped (symmetric) workspaces for in-kernel collectives over NVLink.

A :class:`SymmetricWorkspace` owns, for one process group, buffers that every
member maps into its address space (allocated through PyTorch's symmetric
memory, which exchanges the VMM handles over the process group), the table of
peer pointers, per-peer signal pads used by the kernels' bounded-wait
barriers, the NVLS multicast address when the switch supports it, and a
host-readable status word that a kernel sets when a wait times out.  Native
kernels in :mod:`hybrid_training.ops.comm` take these pointers directly.
"""

from __future__ import annotations

from typing import Any

import torch

from ..errors import CollectiveError, KernelError, format_error
from ..logging import get_logger
from .groups import GroupHandle

__all__ = ["SymmetricWorkspace"]

_LOG = get_logger(__name__)


class SymmetricWorkspace:
    """Symmetric buffers + signal pads for one group (see the module docstring)."""

    # Bytes of each allocation's signal pad.  The kernels' barriers use one 32-bit slot per
    # (block, peer) in the upper half, so 64 KB allows 1024 blocks at 8 ranks (one per SM needs 148).
    SIGNAL_PAD_BYTES = 64 * 1024

    def __init__(self, group: GroupHandle, device: torch.device) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        if symm_mem.get_signal_pad_size() < self.SIGNAL_PAD_BYTES:
            symm_mem.set_signal_pad_size(self.SIGNAL_PAD_BYTES)

        self.group = group
        self.device = device
        self._symm = symm_mem
        self._allocations: list[tuple[torch.Tensor, Any]] = []
        self.status = torch.zeros(4, dtype=torch.int32, device=device)
        self._barrier_epoch = 0

    @classmethod
    def create(cls, group: GroupHandle, device: torch.device) -> SymmetricWorkspace | None:
        """A workspace, or ``None`` when in-kernel collectives are unavailable (CPU, trivial group, no peer access)."""
        if group.is_trivial or device.type != "cuda" or group.process_group is None:
            return None
        try:
            return cls(group, device)
        except Exception as exc:  # pragma: no cover - depends on the machine
            _LOG.warning("symmetric memory unavailable for group %r (%s); using NCCL", group.name, exc)
            return None

    def allocate(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        """A zero-initialised tensor in peer-mapped memory (collective: every member must call it)."""
        t = self._symm.empty(numel, dtype=dtype, device=self.device)
        # Zero before the handle exchange and wait for it: once any rank returns from the
        # rendezvous (a collective), every rank's zeroing is complete, so a peer's first write
        # into this buffer can never be overwritten by the owner's initialisation.
        t.zero_()
        torch.cuda.synchronize(self.device)
        handle = self._symm.rendezvous(t, self.group.process_group)
        self._allocations.append((t, handle))
        return t

    def handle_of(self, tensor: torch.Tensor) -> Any:
        ptr = tensor.untyped_storage().data_ptr()
        for t, h in self._allocations:
            if t.untyped_storage().data_ptr() == ptr:
                return h
        raise CollectiveError(format_error("symmetric.handle_of", "tensor was not allocated from this workspace",
                                           expected="a tensor returned by allocate()", observed=hex(ptr),
                                           resolution="allocate the buffer with SymmetricWorkspace.allocate"))

    def check_status(self) -> None:
        """Raise :class:`KernelError` if a kernel on this workspace reported a timed-out wait."""
        code = int(self.status[0].item())
        if code != 0:
            where = int(self.status[1].item())
            self.status.zero_()
            raise KernelError(format_error("symmetric.check_status", "an in-kernel collective timed out waiting for a peer",
                                           rank=self.group.global_rank, expected="status 0", observed=f"status {code} at stage {where}",
                                           resolution="a peer rank stopped issuing collectives; check every rank's log"))

    def close(self) -> None:
        self._allocations.clear()
