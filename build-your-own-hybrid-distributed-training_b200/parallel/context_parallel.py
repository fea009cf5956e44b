"""Context parallelism: all-gather attention on the native kernel, ring attention and Ulysses
all-to-all attention.

All-gather form (:func:`gathered_attention`, CUDA): every rank gathers the keys and values of the
whole sequence, places its own queries at their positions in a packed full-sequence tensor, and
runs the tcgen05 flash kernel over its query window only (the window's rows against every key,
causal by global position); the backward kernels produce dQ for the window and dK / dV for every
key from the window's queries, and a reduce-scatter returns each key chunk's gradient sum to its
owner.

Ring attention is the form whose memory per rank does not grow with the sequence.

The ranks of a sequence group hold consecutive chunks of the sequence.  Each rank keeps its
query chunk and passes key/value chunks around the ring (send to ``r + 1``, receive from
``r - 1``), merging each chunk's contribution into running softmax statistics (maximum,
normaliser, weighted sum), so no rank ever holds more than two key/value chunks or a score
block larger than ``S/C x S/C``.  Under causal masking a chunk from a later position block
contributes nothing and its computation is skipped (it is still passed on).

The backward pass recomputes the probabilities from the saved log-sum-exp; the key/value
chunks travel the ring again together with their gradient accumulators, which return to
their owners after a full turn.

The reference describes ring attention (``docs/06_sequence_parallelism.md:239-245``) and
provides its primitives (``topology.py:377``, ``collectives.py:669-750``) but does not
implement it.  This implementation is plain PyTorch math over the collective wrappers' point-
to-point transfers (Gloo or NCCL); it is the memory-bounded alternative to the all-gather form
in :class:`hybrid_training.models.transformer.TensorParallelAttention`.
"""

from __future__ import annotations

import math
from typing import Any

import torch

from ..autograd.collectives import all_gather_along_dim, reduce_scatter_along_dim
from ..distributed.collectives import ReduceOp, recv_tensor, send_tensor
from ..distributed.groups import GroupHandle

__all__ = ["gathered_attention", "gathered_attention_supported", "ring_attention", "ulysses_attention"]


def _ring_pass(tensors: list[torch.Tensor], group: GroupHandle) -> list[torch.Tensor]:
    """Send every tensor to the next rank of the ring and return the ones from the previous rank.

    Even ranks send first and odd ranks receive first, so blocking transfers cannot deadlock
    (with an odd group size the last rank is odd-indexed or the first is even; either way one
    side of every pair is receiving).
    """
    me, n = group.local_rank, group.size
    nxt, prv = (me + 1) % n, (me - 1) % n
    out = [torch.empty_like(t) for t in tensors]
    if me % 2 == 0:
        for t in tensors:
            send_tensor(t.contiguous(), group, destination_local_rank=nxt)
        for o in out:
            recv_tensor(o, group, source_local_rank=prv)
    else:
        for o in out:
            recv_tensor(o, group, source_local_rank=prv)
        for t in tensors:
            send_tensor(t.contiguous(), group, destination_local_rank=nxt)
    return out


def _scores(q: torch.Tensor, k: torch.Tensor, scale: float, diagonal: bool) -> torch.Tensor:
    s = (q @ k.transpose(-1, -2)) * scale
    if diagonal:
        n = s.shape[-1]
        s = s.masked_fill(torch.ones(n, n, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
    return s


class _RingAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, group: GroupHandle, causal: bool) -> torch.Tensor:
        # q: [B, H, L, D]; k, v: [B, H, L, D] (key/value heads already expanded to H), fp32
        me, n = group.local_rank, group.size
        scale = 1.0 / math.sqrt(q.shape[-1])
        m = torch.full(q.shape[:-1], float("-inf"), dtype=q.dtype, device=q.device)
        l = torch.zeros_like(m)
        acc = torch.zeros_like(q)
        kv = [k, v]
        for step in range(n):
            src = (me - step) % n  # owner of the chunk held at this step
            if not (causal and src > me):
                s = _scores(q, kv[0], scale, causal and src == me)
                m_new = torch.maximum(m, s.amax(-1))
                alpha = torch.exp(m - m_new)
                p = torch.exp(s - m_new[..., None])
                l = l * alpha + p.sum(-1)
                acc = acc * alpha[..., None] + p @ kv[1]
                m = m_new
            if step < n - 1:
                kv = _ring_pass(kv, group)
        out = acc / l[..., None]
        lse = m + torch.log(l)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.group, ctx.causal = group, causal
        return out

    @staticmethod
    def backward(ctx: Any, dout: torch.Tensor) -> tuple[Any, ...]:
        q, k, v, out, lse = ctx.saved_tensors
        group, causal = ctx.group, ctx.causal
        me, n = group.local_rank, group.size
        scale = 1.0 / math.sqrt(q.shape[-1])
        dout = dout.contiguous()
        delta = (dout * out).sum(-1)
        dq = torch.zeros_like(q)
        travel = [k, v, torch.zeros_like(k), torch.zeros_like(v)]  # chunk and its gradient accumulators
        for step in range(n):
            src = (me - step) % n
            kc, vc, dk, dv = travel
            if not (causal and src > me):
                p = torch.exp(_scores(q, kc, scale, causal and src == me) - lse[..., None])
                dv = dv + p.transpose(-1, -2) @ dout
                ds = p * (dout @ vc.transpose(-1, -2) - delta[..., None])
                dq = dq + (ds @ kc) * scale
                dk = dk + (ds.transpose(-1, -2) @ q) * scale
            # a full turn brings every chunk (and its accumulated gradient) back to its owner
            travel = _ring_pass([kc, vc, dk, dv], group)
        return dq, travel[2], travel[3], None, None


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, group: GroupHandle, *, causal: bool = True) -> torch.Tensor:
    """Attention of this rank's query chunk over the whole sequence, keys/values passed around the ring.

    ``q``, ``k``, ``v``: ``[B, H, L, D]`` with ``L`` the local chunk length (equal on every rank)
    and key/value heads already repeated to ``H``.  Returns ``[B, H, L, D]`` in ``q``'s dtype;
    the arithmetic runs in fp32.
    """
    dtype = q.dtype
    if group.size == 1:
        s = _scores(q.float(), k.float(), 1.0 / math.sqrt(q.shape[-1]), causal)
        return (torch.softmax(s, -1) @ v.float()).to(dtype)
    return _RingAttention.apply(q.float().contiguous(), k.float().contiguous(), v.float().contiguous(), group, causal).to(dtype)


# ------------------------------------------------------------------------------------------------
# Ulysses: all-to-all between sequence chunks and head groups.
# ------------------------------------------------------------------------------------------------
class _AllToAll(torch.autograd.Function):
    """Equal-split all-to-all along dim 0; its adjoint is the same exchange applied to the gradient."""

    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, group: GroupHandle) -> torch.Tensor:
        from ..distributed.collectives import all_to_all_tensor

        ctx.group = group
        return all_to_all_tensor(x.contiguous(), group)

    @staticmethod
    def backward(ctx: Any, grad: torch.Tensor) -> tuple[Any, ...]:
        from ..distributed.collectives import all_to_all_tensor

        return all_to_all_tensor(grad.contiguous(), ctx.group), None


def ulysses_attention(qkv: torch.Tensor, num_heads: int, num_kv_heads: int, head_dim: int, group: GroupHandle, *,
                      causal: bool = True) -> torch.Tensor:
    """Context-parallel attention by re-sharding from sequence chunks to head groups and back.

    ``qkv``: ``[B, L, (H + 2 Hkv) * D]``, this rank's chunk of ``L = S / C`` consecutive positions
    (rotary positions already applied with the global offset).  One all-to-all gives every rank
    the whole sequence for ``H / C`` query heads and ``Hkv / C`` key/value heads; ordinary causal
    attention runs on that (the native flash kernel on CUDA, so context parallelism uses the same
    tensor-core kernel as the single-GPU path); a second all-to-all returns each rank's positions
    for all heads.  Returns ``[B, L, H * D]``.  Needs ``H`` and ``Hkv`` divisible by ``C``.

    The reference describes this scheme (``docs/06_sequence_parallelism.md:247-251``) and
    provides ``all_to_all_tensor`` (``distributed/collectives.py:614-666``) without using it.
    """
    from .. import ops

    c = group.size
    b, length, _ = qkv.shape
    h, hkv, d = num_heads, num_kv_heads, head_dim
    hl, hkvl = h // c, hkv // c
    if c == 1:
        return ops.attention(qkv, h, hkv, d, causal=causal)
    q = qkv[..., : h * d].reshape(b, length, c, hl * d)
    k = qkv[..., h * d:(h + hkv) * d].reshape(b, length, c, hkvl * d)
    v = qkv[..., (h + hkv) * d:].reshape(b, length, c, hkvl * d)
    # [C (destination head group), B, L, local packed qkv] -> exchange -> [C (source chunk), B, L, ...]
    send = torch.cat([q, k, v], dim=-1).permute(2, 0, 1, 3)
    recv = _AllToAll.apply(send, group)
    full = recv.permute(1, 0, 2, 3).reshape(b, c * length, (hl + 2 * hkvl) * d)  # the whole sequence, local heads
    context = ops.attention(full.contiguous(), hl, hkvl, d, causal=causal)      # [B, S, hl * d]
    back = context.reshape(b, c, length, hl * d).permute(1, 0, 2, 3)          # [C (destination chunk), B, L, hl*d]
    mine = _AllToAll.apply(back, group)                                        # [C (source head group), B, L, hl*d]
    return mine.permute(1, 2, 0, 3).reshape(b, length, h * d)


def gathered_attention_supported(local_len: int, head_dim: int) -> bool:
    """Whether :func:`gathered_attention` applies: windows start on 128-row tiles, D is 64 or 128."""
    return local_len % 128 == 0 and head_dim in (64, 128)


class _GatheredAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, qkv: torch.Tensor, h: int, hkv: int, d: int, group: GroupHandle, causal: bool) -> torch.Tensor:
        from ..ops.attention import attention_window_forward

        b, local, width = qkv.shape
        begin, total = group.local_rank * local, local * group.size
        kv = all_gather_along_dim(qkv[..., h * d:].contiguous(), group, 1)  # [B, S, 2 * Hkv * D]
        full = torch.empty(b, total, width, dtype=qkv.dtype, device=qkv.device)
        full[..., h * d:] = kv
        full[:, begin:begin + local, : h * d] = qkv[..., : h * d]  # other ranks' query columns stay unread
        out_full, lse = attention_window_forward(full, h, hkv, d, begin, local, causal)
        ctx.save_for_backward(full, out_full, lse)
        ctx.dims = (h, hkv, d, causal, begin, local, group)
        return out_full[:, begin:begin + local].contiguous()

    @staticmethod
    def backward(ctx: Any, dout: torch.Tensor) -> tuple[Any, ...]:
        from ..ops.attention import attention_window_backward

        full, out_full, lse = ctx.saved_tensors
        h, hkv, d, causal, begin, local, group = ctx.dims
        dqkv = attention_window_backward(full, out_full, lse, dout.contiguous(), h, hkv, d, begin, local, causal)
        dkv = reduce_scatter_along_dim(dqkv[..., h * d:].contiguous(), group, 1, op=ReduceOp.SUM)  # this rank's keys
        dq = dqkv[:, begin:begin + local, : h * d]
        return torch.cat([dq, dkv], dim=-1), None, None, None, None, None


def gathered_attention(qkv: torch.Tensor, num_heads: int, num_kv_heads: int, head_dim: int, group: GroupHandle, *,
                       causal: bool = True) -> torch.Tensor:
    """Context-parallel attention of this rank's chunk ``qkv`` ``[B, S/C, W]`` (positions ``r S/C ..``)
    against the keys of the whole sequence, on the native flash kernels (see the module docstring)."""
    return _GatheredAttention.apply(qkv, num_heads, num_kv_heads, head_dim, group, causal)
