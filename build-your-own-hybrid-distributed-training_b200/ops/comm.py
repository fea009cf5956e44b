"""Collectives computed inside native kernels over NVLink peer memory.

``bucket_all_reduce`` averages one DDP gradient bucket across the data-parallel
group with a single kernel that reads the peers' buffers directly (two-shot
reduce-scatter + all-gather over P2P loads, or, when the NVLink switch offers
a multicast address and ``HT_NVLS=1``, one ``multimem.ld_reduce`` /
``multimem.st`` pass), folding the ``1/G`` scale into the reduction.  Its
input must live in a :class:`~hybrid_training.distributed.symmetric.SymmetricWorkspace`
allocation (DDP allocates its flat gradient buffer there).  Every wait in the
kernel is bounded; a timeout sets the workspace status word, which
``SymmetricWorkspace.check_status`` turns into a :class:`KernelError`.

``fsdp_reduce_scatter_adamw`` is the FSDP gradient path in one kernel: each rank
sums its shard of the unit's gradient over the peers' staging buffers, scales
it, zeroes the padding and applies AdamW to its fp32 master shard, writing the
bf16 copy that ``fsdp_all_gather`` (a P2P copy of every peer's bf16 shard into
the local full buffer) reads in the next forward.

The tensor-parallel fused paths (all-gather inside the first GEMM of a
column-parallel layer, reduce-scatter inside the GEMM of a row-parallel layer)
are exposed as :func:`all_gather_linear` / :func:`linear_reduce_scatter`;
:data:`HAS_FUSED_TENSOR_PARALLEL` tells the layers whether to use them.
"""

from __future__ import annotations

import os
from typing import Any

import torch

from ._ext import extension

__all__ = ["HAS_FUSED_TENSOR_PARALLEL", "all_gather_linear", "bucket_all_reduce", "can_fuse_all_reduce",
           "column_linear_reduced_grad", "linear_all_reduce", "nvls_available", "can_fuse_sequence_parallel",
           "fsdp_all_gather", "fsdp_reduce_scatter_adamw", "linear_reduce_scatter"]

HAS_FUSED_TENSOR_PARALLEL = True
_TIMEOUT_S = float(os.environ.get("HT_COLLECTIVE_TIMEOUT_S", "30"))


def _slots(handle: Any, world: int) -> tuple[int, int]:
    """(first signal-pad slot used here, max blocks): the upper half of each pad is reserved for these kernels."""
    slots = int(handle.signal_pad_size) // 4
    base = slots // 2
    return base, max(1, (slots - base) // world)


def nvls_available(workspace: Any, flat: torch.Tensor) -> bool:
    """Whether ``flat``'s allocation has an NVLink-switch multicast address (NVLS)."""
    return int(getattr(workspace.handle_of(flat), "multicast_ptr", 0) or 0) != 0


def bucket_all_reduce(workspace: Any, flat: torch.Tensor, start: int, numel: int, scale: float, *,
                      wide: bool = True, peer_slots: int = 0) -> torch.Tensor:
    """Average ``flat[start:start+numel]`` over the workspace's group in place; returns the status tensor.

    ``wide=False`` launches the narrow shape that runs beside a persistent GEMM (for buckets
    reduced while the backward pass is still computing); ``wide=True`` the full-width shape for a
    reduction that has the GPU to itself.  ``HT_NVLS=1`` selects the NVLink-switch reduction where
    the allocation has a multicast address; otherwise the two-shot P2P kernel runs.  ``peer_slots``
    (2, 4 or 8) selects a kernel instantiation for at least that many peers (tests only).
    """
    handle = workspace.handle_of(flat)
    world = workspace.group.size
    base, max_blocks = _slots(handle, world)
    mc = int(getattr(handle, "multicast_ptr", 0) or 0) if os.environ.get("HT_NVLS", "0") == "1" else 0
    extension().bucket_all_reduce(flat, list(handle.buffer_ptrs), list(handle.signal_pad_ptrs), mc, int(start), int(numel),
                                  float(scale), int(handle.rank), base, max_blocks, workspace.status, _TIMEOUT_S,
                                  bool(wide), int(peer_slots))
    return workspace.status


def fsdp_reduce_scatter_adamw(workspace: Any, staging: torch.Tensor, shard16: torch.Tensor, *, shard: int, valid: int,
                              scale: float, param: torch.Tensor, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor,
                              hyper: torch.Tensor, betas: tuple[float, float], eps: float, weight_decay: float,
                              grad_out: torch.Tensor | None = None, slice_index: int | None = None) -> torch.Tensor:
    """Reduce-scatter the unit gradient in every peer's ``staging`` and apply AdamW to this rank's shard.

    ``staging`` (bf16 or fp32, the unit's padded gradient) must be an allocation of ``workspace``,
    whose group is the set of ranks whose gradients are summed: the shard group, or under hybrid
    sharding the data-parallel x shard group, with ``slice_index`` this rank's index in the shard
    group (default: its rank in ``workspace``).  ``shard16`` (bf16, ``shard`` elements) receives
    the updated shard for the next all-gather; ``param`` / ``exp_avg`` /
    ``exp_avg_sq`` are this rank's fp32 master shard and moments; ``hyper`` is the optimizer's
    device vector ``[lr, step, grad_scale, skip]``.  Elements at local index ``>= valid`` are
    padding and get a zero gradient.  ``grad_out`` (fp32, optional) receives the reduced shard
    gradient.  Returns the workspace status word (non-zero after a timed-out peer wait).
    """
    handle = workspace.handle_of(staging)
    world = workspace.group.size
    base, max_blocks = _slots(handle, world)
    extension().fsdp_reduce_scatter_adamw(staging, list(handle.buffer_ptrs), list(handle.signal_pad_ptrs), int(handle.rank),
                                          int(shard), int(valid), float(scale), param, exp_avg, exp_avg_sq, shard16, grad_out,
                                          hyper, float(betas[0]), float(betas[1]), float(eps), float(weight_decay), base,
                                          max_blocks, workspace.status, _TIMEOUT_S, -1 if slice_index is None else int(slice_index))
    return workspace.status


def fsdp_all_gather(workspace: Any, shard16: torch.Tensor, out: torch.Tensor, *, copy_engine: bool = False) -> None:
    """Copy every peer's bf16 shard (``shard16``, a workspace allocation) into ``out`` (rank order).

    ``copy_engine=False`` runs the P2P load kernel; ``True`` issues one peer ``cudaMemcpyAsync``
    per rank, which occupies no SMs and so overlaps a concurrently running compute kernel.
    """
    handle = workspace.handle_of(shard16)
    fn = extension().fsdp_all_gather_copy_engine if copy_engine else extension().fsdp_all_gather
    fn(list(handle.buffer_ptrs), out, int(shard16.numel()), int(handle.rank))


class _TensorParallelSites:
    """Per-group state of the fused tensor-parallel collectives.

    * one peer-mapped int32 flag array ``[site][8]``: peer ``p`` writes the epoch it published
      for a call site into word ``[site][p]`` of every other rank;
    * one local int32 counter pair per site (epoch, completed CTAs), advanced on the device so
      that replaying a captured CUDA graph advances it too;
    * peer-mapped shard / receive buffers per call site, allocated on first use (every rank
      reaches the same call sites in the same order, which keeps the collective allocation
      and the site numbering aligned across ranks).
    """

    MAX_SITES = 512

    def __init__(self, workspace: Any) -> None:
        self.workspace = workspace
        self.flags = workspace.allocate(self.MAX_SITES * 8, torch.int32)
        self.flag_ptrs = [int(p) for p in workspace.handle_of(self.flags).buffer_ptrs]
        self.counters = torch.zeros(self.MAX_SITES * 2, dtype=torch.int32, device=self.flags.device)
        self.sites: dict[tuple[Any, str], int] = {}
        self.buffers: dict[tuple[Any, str], tuple[torch.Tensor, list[int]]] = {}
        self.local: dict[tuple[Any, str], torch.Tensor] = {}
        self.rank = int(workspace.group.local_rank)
        self.world = int(workspace.group.size)

    def site(self, owner: Any, kind: str) -> int:
        key = (owner, kind)
        if key not in self.sites:
            if len(self.sites) >= self.MAX_SITES:
                raise RuntimeError("too many fused tensor-parallel call sites")
            self.sites[key] = len(self.sites)
        return self.sites[key]

    def buffer(self, owner: Any, kind: str, shape: tuple[int, ...]) -> tuple[torch.Tensor, list[int]]:
        key = (owner, kind)
        numel = 1
        for d in shape:
            numel *= d
        hit = self.buffers.get(key)
        if hit is None or hit[0].numel() != numel:
            t = self.workspace.allocate(numel, torch.bfloat16)
            hit = (t, [int(p) for p in self.workspace.handle_of(t).buffer_ptrs])
            self.buffers[key] = hit
        return hit[0].view(shape), hit[1]


    def local_buffer(self, owner: Any, kind: str, shape: tuple[int, ...], dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """A persistent buffer of this rank only (gathered copies, block flags); flags start at zero."""
        key = (owner, kind)
        t = self.local.get(key)
        numel = 1
        for d in shape:
            numel *= d
        if t is None or t.numel() != numel or t.dtype != dtype:
            t = torch.zeros(numel, dtype=dtype, device=self.flags.device)
            self.local[key] = t
        return t.view(shape)


_SITES: dict[int, _TensorParallelSites] = {}


def _note(operation: str, st: _TensorParallelSites, tensor: torch.Tensor) -> None:
    """Count a fused collective for :func:`~hybrid_training.distributed.collectives.observe_collectives`."""
    from ..distributed.collectives import record_collective

    record_collective(None, operation, st.workspace.group.name, num_bytes=tensor.numel() * tensor.element_size())


def _sites(workspace: Any) -> _TensorParallelSites:
    st = _SITES.get(id(workspace))
    if st is None:
        st = _SITES[id(workspace)] = _TensorParallelSites(workspace)
    return st


def can_fuse_sequence_parallel(x: torch.Tensor, group: Any, *, sharded_rows: int, features: tuple[int, ...]) -> bool:
    """Whether the fused kernels cover this call: bf16 on CUDA, 2..8 ranks, 128-row shards, 16-byte rows."""
    return (x.is_cuda and x.dtype == torch.bfloat16 and 2 <= group.size <= 8 and sharded_rows % 128 == 0
            and all(f % 64 == 0 for f in features))


class _AllGatherLinear(torch.autograd.Function):
    """``Y = AllGather_seq(X) W^T (+ b, GELU)`` with the gather inside the GEMM's operand loads."""

    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, workspace: Any, owner: Any,
                activation: str | None) -> torch.Tensor:
        from .linear import EPI_GELU, EPI_PLAIN, compute_weight

        st = _sites(workspace)
        ext = extension()
        b, r, k = x.shape
        w = compute_weight(weight, x.dtype)
        n = w.shape[0]
        slot, ptrs = st.buffer(owner, "ag.x", (b, r, k))
        slot.copy_(x)
        site = st.site(owner, "ag")
        y = torch.empty(b * r * st.world, n, dtype=x.dtype, device=x.device)
        pre = torch.empty_like(y) if activation == "gelu" else None
        gathered = st.local_buffer(owner, "ag.gathered", (b, r * st.world, k))
        flags = st.local_buffer(owner, "ag.blocks", (b * r * st.world // 128 * (k // 64),), torch.int32)
        ext.gemm_collective(slot, w, y, bias, pre, False, False, EPI_GELU if pre is not None else EPI_PLAIN, 0.0,
                            1, ptrs, 0, [], 0, [], st.flags, st.flag_ptrs, st.counters, site, 1, st.rank, _TIMEOUT_S,
                            gathered, flags)
        _note("all_gather_gemm", st, x)
        ctx.save_for_backward(w, pre)
        ctx.st, ctx.owner, ctx.site, ctx.shape = st, owner, site, (b, r, k)
        ctx.weight, ctx.bias = weight, bias
        return y.view(b, r * st.world, n)

    @staticmethod
    def backward(ctx: Any, dy: torch.Tensor) -> tuple[Any, ...]:
        from .grads import deliver_grad
        from .linear import EPI_PLAIN, _column_sum, gelu_backward, gemm

        w, pre = ctx.saved_tensors
        st, owner = ctx.st, ctx.owner
        ext = extension()
        b, r, k = ctx.shape
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        g = gelu_backward(dy2, pre) if pre is not None else dy2
        dx = None
        if ctx.needs_input_grad[0]:
            recv, rptrs = st.buffer(owner, "ag.dx_recv", (st.world, b, r, k))
            site = st.site(owner, "ag.rs")
            ext.gemm_collective(g, w, recv, None, None, False, True, EPI_PLAIN, 0.0, 0, [], 0, [], 1, rptrs,
                                st.flags, st.flag_ptrs, st.counters, site, 1, st.rank, _TIMEOUT_S, None, None)
            dx = torch.empty(b, r, k, dtype=dy.dtype, device=dy.device)
            ext.reduce_scatter_sum(recv, dx, st.flags, st.counters, site, st.rank, _TIMEOUT_S)
            _note("gemm_reduce_scatter", st, recv)
        gathered = st.local_buffer(owner, "ag.gathered", (b, r * st.world, k)).view(-1, k)
        weight, bias = ctx.weight, ctx.bias

        def wgrad(out: torch.Tensor, beta: float) -> None:
            gemm(g, gathered, out=out, a_mn_major=True, b_mn_major=True, beta=beta)

        dw = None
        if ctx.needs_input_grad[1]:
            value = None
            if getattr(weight, "main_grad", None) is None:
                value = torch.empty(weight.shape, dtype=torch.float32, device=dy.device)
                wgrad(value, 0.0)
                value = value.to(weight.dtype)
            dw = deliver_grad(weight, compute=wgrad if value is None else None, value=value)
        db = None
        if bias is not None and ctx.needs_input_grad[2]:
            db = deliver_grad(bias, compute=lambda out, beta: _column_sum(g, out, beta),
                              value=None if getattr(bias, "main_grad", None) is not None else _column_sum(g).to(bias.dtype))
        return dx, dw, db, None, None, None


class _LinearReduceScatter(torch.autograd.Function):
    """``out = ReduceScatter_seq(X W^T)`` with the scatter inside the GEMM epilogue."""

    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, weight: torch.Tensor, workspace: Any, owner: Any) -> torch.Tensor:
        from .linear import EPI_PLAIN, compute_weight

        st = _sites(workspace)
        ext = extension()
        b, s, kr = x.shape
        r = s // st.world
        w = compute_weight(weight, x.dtype)
        n = w.shape[0]
        x2 = x.reshape(b * s, kr).contiguous()
        recv, rptrs = st.buffer(owner, "rs.recv", (st.world, b, r, n))
        site = st.site(owner, "rs")
        ext.gemm_collective(x2, w, recv, None, None, False, False, EPI_PLAIN, 0.0, 0, [], 0, [], 1, rptrs,
                            st.flags, st.flag_ptrs, st.counters, site, 1, st.rank, _TIMEOUT_S, None, None)
        out = torch.empty(b, r, n, dtype=x.dtype, device=x.device)
        ext.reduce_scatter_sum(recv, out, st.flags, st.counters, site, st.rank, _TIMEOUT_S)
        _note("gemm_reduce_scatter", st, recv)
        ctx.save_for_backward(x2, w)
        ctx.st, ctx.owner, ctx.dims, ctx.weight = st, owner, (b, s, kr, n), weight
        return out

    @staticmethod
    def backward(ctx: Any, dout: torch.Tensor) -> tuple[Any, ...]:
        from .grads import deliver_grad
        from .linear import EPI_PLAIN, gemm

        x2, w = ctx.saved_tensors
        st, owner = ctx.st, ctx.owner
        ext = extension()
        b, s, kr, n = ctx.dims
        r = s // st.world
        slot, ptrs = st.buffer(owner, "rs.dout", (b, r, n))
        slot.copy_(dout.reshape(b, r, n))
        site = st.site(owner, "rs.ag")
        gathered = st.local_buffer(owner, "rs.gathered", (b, s, n))
        flags = st.local_buffer(owner, "rs.blocks", (b * s // 128 * (n // 64),), torch.int32)
        # dX = AllGather(dout) W: the gather happens inside this GEMM and leaves the gathered copy
        # that the weight gradient reads.
        dx = torch.empty(b * s, kr, dtype=dout.dtype, device=dout.device)
        ext.gemm_collective(slot, w, dx, None, None, False, True, EPI_PLAIN, 0.0, 1, ptrs, 0, [], 0, [],
                            st.flags, st.flag_ptrs, st.counters, site, 1, st.rank, _TIMEOUT_S, gathered, flags)
        _note("all_gather_gemm", st, slot)
        weight = ctx.weight
        g2 = gathered.view(b * s, n)

        def wgrad(out: torch.Tensor, beta: float) -> None:
            gemm(g2, x2, out=out, a_mn_major=True, b_mn_major=True, beta=beta)

        dw = None
        if ctx.needs_input_grad[1]:
            value = None
            if getattr(weight, "main_grad", None) is None:
                value = torch.empty(weight.shape, dtype=torch.float32, device=dout.device)
                wgrad(value, 0.0)
                value = value.to(weight.dtype)
            dw = deliver_grad(weight, compute=wgrad if value is None else None, value=value)
        return dx.view(b, s, kr), dw, None, None


def _sum_over_group(st: _TensorParallelSites, owner: Any, kind: str, rows: int, cols: int,
                    produce: Any) -> torch.Tensor:
    """``produce(out)`` writes this rank's fp32 partial ``[rows, cols]`` straight into a peer-mapped
    buffer (the GEMM's TMA-store epilogue); the two-shot in-kernel NVLink all-reduce then sums it in
    place across the group.  Returns the sum (a view of the buffer, valid until the next call of
    this site)."""
    key = (owner, kind)
    buf = st.local.get(key)
    if buf is None or buf.numel() != rows * cols:
        buf = st.workspace.allocate(rows * cols, torch.float32)
        st.local[key] = buf
    out = buf.view(rows, cols)
    produce(out)
    bucket_all_reduce(st.workspace, buf, 0, rows * cols, 1.0, wide=True)
    _note("gemm_all_reduce", st, out)
    return out


class _LinearAllReduce(torch.autograd.Function):
    """Row-parallel ``out = AllReduce(X W_r^T)`` (tensor parallelism without sequence parallelism).

    Forward: the GEMM writes its fp32 partial product into peer-mapped memory and the in-kernel
    all-reduce sums it (reference: the ``reduce_from_group`` all-reduce after the row-parallel
    GEMM, ``autograd/collectives.py:192``, ``tensor_parallel.py:456``).  Backward: the output
    gradient is the same on every rank, so the input and weight gradients are local GEMMs.
    """

    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, weight: torch.Tensor, workspace: Any, owner: Any) -> torch.Tensor:
        from .linear import compute_weight, gemm

        st = _sites(workspace)
        lead, k = x.shape[:-1], x.shape[-1]
        x2 = x.reshape(-1, k).contiguous()
        w = compute_weight(weight, x.dtype)
        n = w.shape[0]
        summed = _sum_over_group(st, owner, "ar.out", x2.shape[0], n, lambda out: gemm(x2, w, out=out))
        ctx.save_for_backward(x2, w)
        ctx.weight = weight
        return summed.to(x.dtype).view(*lead, n)

    @staticmethod
    def backward(ctx: Any, dy: torch.Tensor) -> tuple[Any, ...]:
        from .grads import deliver_grad
        from .linear import gemm

        x2, w = ctx.saved_tensors
        weight = ctx.weight
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        dx = gemm(dy2, w, b_mn_major=True).view(*dy.shape[:-1], w.shape[1]) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            dw = deliver_grad(weight, compute=lambda out, beta: gemm(dy2, x2, out=out, a_mn_major=True, b_mn_major=True,
                                                                      beta=beta),
                              value=None if getattr(weight, "main_grad", None) is not None else
                              gemm(dy2, x2, out_dtype=weight.dtype, a_mn_major=True, b_mn_major=True))
        return dx, dw, None, None


class _ColumnLinearReducedGrad(torch.autograd.Function):
    """Column-parallel ``Y = act(X W_r^T + b_r)`` whose input gradient is all-reduced in-kernel.

    Forward: a local GEMM (GELU in its epilogue).  Backward: the input-gradient GEMM writes its fp32
    partial into peer-mapped memory and the in-kernel all-reduce sums it (reference: the
    ``copy_to_group`` adjoint, ``autograd/collectives.py:180``).
    """

    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, workspace: Any, owner: Any,
                gelu: bool) -> torch.Tensor:
        from .linear import EPI_GELU, compute_weight, gemm

        lead, k = x.shape[:-1], x.shape[-1]
        x2 = x.reshape(-1, k).contiguous()
        w = compute_weight(weight, x.dtype)
        y = torch.empty(x2.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
        pre = None
        if gelu:
            pre = torch.empty_like(y)
            gemm(x2, w, out=y, bias=bias, aux=pre, epilogue=EPI_GELU)
        else:
            gemm(x2, w, out=y, bias=bias)
        ctx.save_for_backward(x2, w, pre)
        ctx.weight, ctx.bias, ctx.st, ctx.owner = weight, bias, _sites(workspace), owner
        return y.view(*lead, w.shape[0])

    @staticmethod
    def backward(ctx: Any, dy: torch.Tensor) -> tuple[Any, ...]:
        from .grads import deliver_grad
        from .linear import _column_sum, gelu_backward, gemm

        x2, w, pre = ctx.saved_tensors
        weight, bias = ctx.weight, ctx.bias
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        g = gelu_backward(dy2, pre) if pre is not None else dy2
        dx = None
        if ctx.needs_input_grad[0]:
            summed = _sum_over_group(ctx.st, ctx.owner, "ar.dx", g.shape[0], w.shape[1],
                                     lambda out: gemm(g, w, out=out, b_mn_major=True))
            dx = summed.to(dy.dtype).view(*dy.shape[:-1], w.shape[1])
        dw = db = None
        if ctx.needs_input_grad[1]:
            dw = deliver_grad(weight, compute=lambda out, beta: gemm(g, x2, out=out, a_mn_major=True, b_mn_major=True,
                                                                      beta=beta),
                              value=None if getattr(weight, "main_grad", None) is not None else
                              gemm(g, x2, out_dtype=weight.dtype, a_mn_major=True, b_mn_major=True))
        if bias is not None and ctx.needs_input_grad[2]:
            db = deliver_grad(bias, compute=lambda out, beta: _column_sum(g, out, beta),
                              value=None if getattr(bias, "main_grad", None) is not None else _column_sum(g).to(bias.dtype))
        return dx, dw, db, None, None, None


def can_fuse_all_reduce(x: torch.Tensor, group: Any, *, features: tuple[int, ...]) -> bool:
    """Whether the in-kernel all-reduce covers this tensor-parallel call: bf16 on CUDA, 2..8 ranks, 16-byte rows."""
    return x.is_cuda and x.dtype == torch.bfloat16 and 2 <= group.size <= 8 and all(f % 8 == 0 for f in features)


def linear_all_reduce(x: torch.Tensor, weight: torch.Tensor, workspace: Any, group: Any, *,
                      owner: Any = None) -> torch.Tensor | None:
    """Row-parallel linear (no sequence parallelism) with its output summed in-kernel; ``None`` when not applicable."""
    if not can_fuse_all_reduce(x, group, features=(x.shape[-1], weight.shape[0])):
        return None
    return _LinearAllReduce.apply(x, weight, workspace, owner if owner is not None else id(weight))


def column_linear_reduced_grad(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, workspace: Any, group: Any,
                               *, activation: str | None = None, owner: Any = None) -> torch.Tensor | None:
    """Column-parallel linear (no sequence parallelism) whose input gradient is summed in-kernel; ``None``
    when not applicable."""
    if activation not in (None, "gelu") or not can_fuse_all_reduce(x, group, features=(x.shape[-1], weight.shape[0])):
        return None
    return _ColumnLinearReducedGrad.apply(x, weight, bias, workspace, owner if owner is not None else id(weight),
                                          activation == "gelu")


def all_gather_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, workspace: Any, group: Any, *,
                      activation: str | None = None, owner: Any = None) -> torch.Tensor | None:
    """Column-parallel linear on a sequence-sharded ``x`` [B, S/T, K]; ``None`` when the fused kernel does not apply."""
    if activation not in (None, "gelu") or x.dim() != 3:
        return None
    if not can_fuse_sequence_parallel(x, group, sharded_rows=x.shape[1], features=(x.shape[2], weight.shape[0])):
        return None
    from ..utils.tracing import trace_range

    with trace_range("tp/all-gather GEMM"):
        return _AllGatherLinear.apply(x.contiguous(), weight, bias, workspace, owner if owner is not None else id(weight),
                                      activation)


def linear_reduce_scatter(x: torch.Tensor, weight: torch.Tensor, workspace: Any, group: Any, *, owner: Any = None) -> torch.Tensor | None:
    """Row-parallel linear whose output is reduce-scattered along the sequence; ``None`` when not applicable."""
    if x.dim() != 3 or x.shape[1] % group.size:
        return None
    if not can_fuse_sequence_parallel(x, group, sharded_rows=x.shape[1] // group.size, features=(x.shape[2], weight.shape[0])):
        return None
    from ..utils.tracing import trace_range

    with trace_range("tp/GEMM reduce-scatter"):
        return _LinearReduceScatter.apply(x.contiguous(), weight, workspace, owner if owner is not None else id(weight))
