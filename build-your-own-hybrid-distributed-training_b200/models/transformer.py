"""Decoder-only transformer covering GPT-2 and Llama shapes, built from parallel layers.

The module tree and parameter names follow the reference's ``TinyTransformer``
(``src/hybrid_training/models/transformer.py:98-658``): ``token_embedding``,
``position_embedding``, ``blocks.{i}.{input_norm, attention, post_attention_norm,
feed_forward}``, ``final_norm``, ``output_projection``; pre-norm residual
blocks; causal attention; the tensor-parallel plan (vocab-parallel embedding,
column/row layers, sequence parallelism with padding of uneven lengths).

What changes, B200-first:

* q/k/v are **one** column-parallel GEMM (``attention.qkv``) and attention
  reads the packed result directly with a flash kernel (no ``S x S`` scores);
* the residual stream is fp32 and each ``residual + branch`` is fused into the
  following norm (:func:`hybrid_training.ops.add_norm`); branches compute in
  the compute dtype (bf16 under mixed precision) from fp32 master weights;
* GELU is fused into the fc1 GEMM epilogue;
* Llama features: RMSNorm, rotary embeddings, SwiGLU, grouped-query attention,
  no biases;
* with ``targets`` the model returns the mean cross-entropy computed by the
  fused head + vocab-parallel CE op instead of materialising (and, under TP,
  all-gathering) the full logits; without ``targets`` it returns logits
  exactly as the reference does.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..autograd.collectives import copy_to_group, gather_from_sequence_parallel_region, reduce_from_group
from ..config import ModelConfig
from ..distributed.groups import GroupHandle
from ..errors import ConfigurationError, UnsupportedFeatureError, format_error
from ..parallel.sequence_parallel import (
    SEQUENCE_DIM,
    SequenceParallelLayerNorm,
    SequenceParallelRMSNorm,
    SequenceShardInfo,
    gather_sequence,
    local_sequence_slice,
    pad_sequence_dimension,
    scatter_sequence,
    unpad_sequence_dimension,
)
from ..parallel.tensor_parallel import (
    ColumnParallelLinear,
    QKVParallelLinear,
    RowParallelLinear,
    TensorParallelFeedForward,
    VocabParallelEmbedding,
    VocabParallelHead,
    init_linear_parameters,
)
from ..utils.reproducibility import derive_seed, temporary_seed

__all__ = ["LearnedPositionEmbedding", "ParallelPlan", "TensorParallelAttention", "TinyTransformer", "TransformerBlock",
           "build_reference_linear"]


class LearnedPositionEmbedding(nn.Embedding):
    """Learned absolute positions; ``forward(x)`` returns ``x + rows[:S]`` (never a view of the table)."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:  # type: ignore[override]
        return x + self.weight[: x.shape[1]][None].to(x.dtype)


@dataclass(frozen=True)
class ParallelPlan:
    """Which groups the layers of one rank use."""

    tensor_group: GroupHandle
    sequence_group: GroupHandle
    sequence_parallel: bool = False
    vocab_parallel: bool = True
    ring_attention: bool = False  # context parallelism: pass keys/values around the ring instead of all-gathering
    ulysses_attention: bool = False  # context parallelism: all-to-all from sequence chunks to head groups and back

    @property
    def context_parallel(self) -> bool:
        """Sequence parallelism over its own group (``independent`` mode): attention needs every chunk.

        Position-wise layers then run on the local chunk with full weights, and attention
        gathers the keys and values of the whole sequence (see ``TensorParallelAttention``).
        """
        return self.sequence_parallel and self.sequence_group.ranks != self.tensor_group.ranks

    @classmethod
    def single_process(cls) -> ParallelPlan:
        trivial = GroupHandle.trivial("tensor")
        return cls(tensor_group=trivial, sequence_group=trivial, sequence_parallel=False)

    def __post_init__(self) -> None:
        if self.sequence_parallel and self.sequence_group.size == 1:
            raise ConfigurationError(format_error("models.ParallelPlan", "sequence_parallel requested but the sequence group has one member",
                                                  expected="a sequence group with 2 or more ranks", observed=self.sequence_group.size,
                                                  resolution="give the plan a sequence group of 2+ ranks, or turn sequence parallelism off"))
        if self.sequence_parallel and self.sequence_group.ranks != self.tensor_group.ranks and self.tensor_group.size > 1:
            raise UnsupportedFeatureError(format_error(
                "models.ParallelPlan", "sequence parallelism over a group other than the tensor group (independent mode) "
                "combined with tensor parallelism would give attention only the local sequence chunk",
                expected="sequence group == tensor group, or tensor_parallel_size == 1",
                observed=f"sequence {self.sequence_group.ranks} vs tensor {self.tensor_group.ranks}",
                resolution="use sequence_parallel_mode='tensor_group'"))


def _make_norm(config: ModelConfig, plan: ParallelPlan, device: torch.device | None, dtype: torch.dtype | None) -> nn.Module:
    cls = SequenceParallelRMSNorm if config.norm == "rmsnorm" else SequenceParallelLayerNorm
    return cls(config.hidden_size, eps=config.layer_norm_eps, group=plan.tensor_group, sequence_parallel=plan.sequence_parallel,
               device=device, dtype=dtype)


class TensorParallelAttention(nn.Module):
    """Causal (grouped-query) self-attention, heads split over the tensor group."""

    def __init__(self, hidden_size: int, num_heads: int, plan: ParallelPlan, *, num_kv_heads: int | None = None,
                 dropout: float = 0.0, bias: bool = True, causal: bool = True, init_seed: int = 0,
                 device: torch.device | None = None, dtype: torch.dtype | None = None, rope_theta: float | None = None,
                 init_std: float | None = None) -> None:
        super().__init__()
        t = plan.tensor_group.size
        kv = num_kv_heads or num_heads
        if num_heads % t or kv % t:
            raise ConfigurationError(format_error(
                "models.TensorParallelAttention", "the attention heads cannot be split equally over the tensor-parallel ranks",
                rank=plan.tensor_group.global_rank, expected=f"num_heads % {t} == 0 and num_kv_heads % {t} == 0",
                observed=(num_heads, kv), resolution="choose head counts that are multiples of the tensor-parallel size"))
        self.hidden_size, self.num_heads, self.num_kv_heads = hidden_size, num_heads, kv
        self.head_dim = hidden_size // num_heads
        self.heads_per_partition, self.kv_heads_per_partition = num_heads // t, kv // t
        self.causal, self.dropout, self.plan, self.rope_theta = causal, dropout, plan, rope_theta
        self.qkv = QKVParallelLinear(hidden_size, num_heads, kv, self.head_dim, plan.tensor_group, bias=bias,
                                     sequence_parallel=plan.sequence_parallel, init_seed=init_seed, device=device, dtype=dtype,
                                     init_std=init_std)
        self.output = RowParallelLinear(num_heads * self.head_dim, hidden_size, plan.tensor_group, bias=bias, input_is_parallel=True,
                                        sequence_parallel=plan.sequence_parallel, init_seed=derive_seed(init_seed, "attn-o"),
                                        device=device, dtype=dtype, init_std=init_std)
        self._rope_cache: dict[tuple[int, str], tuple[torch.Tensor, torch.Tensor]] = {}

    def _rope(self, seq: int, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
        key = (seq, str(device))
        if key not in self._rope_cache:
            self._rope_cache[key] = ops.rope_tables(seq, self.head_dim, float(self.rope_theta), device)
        return self._rope_cache[key]

    def forward(self, x: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        qkv = self.qkv(x)
        h, hkv, d = self.heads_per_partition, self.kv_heads_per_partition, self.head_dim
        if self.plan.context_parallel:
            return self.output(self._context_parallel(qkv, attention_mask))
        if self.rope_theta is not None:
            cos, sin = self._rope(qkv.shape[1], qkv.device)
            qkv = ops.apply_rope(qkv, cos, sin, h, hkv, d)
        if attention_mask is not None or (self.dropout > 0.0 and self.training):
            context = _explicit_attention(qkv, h, hkv, d, self.causal, attention_mask, self.dropout if self.training else 0.0)
        else:
            context = ops.attention(qkv, h, hkv, d, causal=self.causal)
        return self.output(context)


    def _context_parallel(self, qkv: torch.Tensor, attention_mask: torch.Tensor | None) -> torch.Tensor:
        """Attention of this rank's query chunk against the keys/values of the whole sequence.

        The sequence group's ranks hold consecutive chunks of ``S / C`` positions.  Rotary
        positions are offset by the chunk start; keys and values are all-gathered along the
        sequence (the gather's adjoint reduce-scatters their gradients, so each rank's
        contribution to every key reaches its owner); causal masking compares global
        positions.  On CUDA (chunks of a multiple of 128 positions) the native flash kernels run
        over the rank's query window of a full-sequence packed tensor
        (:func:`~hybrid_training.parallel.context_parallel.gathered_attention`); elsewhere the
        scores are materialised per chunk (``S / C x S``).  This is the all-gather form of context
        parallelism, which the reference describes but does not implement
        (``docs/06_sequence_parallelism.md:234-256``; its ``independent`` mode gives
        attention only the local chunk).  ``context_parallel_algorithm`` selects instead the ring
        with online softmax (memory per rank independent of the sequence) or Ulysses (all-to-all
        to head groups, then the flash kernel over the whole sequence).
        """
        if attention_mask is not None:
            raise UnsupportedFeatureError(format_error(
                "models.attention", "explicit attention masks are not supported with context parallelism",
                expected="attention_mask=None", observed="a mask", resolution="are masked by causality"))
        cp = self.plan.sequence_group
        h, hkv, d = self.heads_per_partition, self.kv_heads_per_partition, self.head_dim
        local = qkv.shape[1]
        offset = cp.local_rank * local
        if self.rope_theta is not None:
            cos, sin = self._rope(local * cp.size, qkv.device)
            qkv = ops.apply_rope(qkv, cos[offset:offset + local].contiguous(), sin[offset:offset + local].contiguous(), h, hkv, d)
        if self.plan.ulysses_attention:
            from ..parallel.context_parallel import ulysses_attention

            if self.dropout > 0.0 and self.training:
                raise UnsupportedFeatureError(format_error(
                    "models.attention", "attention dropout is not implemented by Ulysses attention", expected="dropout=0",
                    observed=self.dropout, resolution="disable attention dropout or use context_parallel_algorithm='all_gather'"))
            if h % cp.size or hkv % cp.size:
                raise UnsupportedFeatureError(format_error(
                    "models.attention", "Ulysses attention gives every rank of the sequence group an equal share of the heads",
                    expected=f"query and key/value head counts divisible by {cp.size}", observed=f"{h} and {hkv}",
                    resolution="use context_parallel_algorithm='ring' or 'all_gather' for this head count"))
            return ulysses_attention(qkv.contiguous(), h, hkv, d, cp, causal=self.causal).to(qkv.dtype)
        q = qkv[..., : h * d]
        if self.plan.ring_attention:
            from ..parallel.context_parallel import ring_attention

            if self.dropout > 0.0 and self.training:
                raise UnsupportedFeatureError(format_error(
                    "models.attention", "attention dropout is not implemented by ring attention", expected="dropout=0",
                    observed=self.dropout, resolution="disable attention dropout or use context_parallel_algorithm='all_gather'"))

            b = q.shape[0]
            qh = q.reshape(b, local, h, d).transpose(1, 2)
            kh = qkv[..., h * d:(h + hkv) * d].reshape(b, local, hkv, d).transpose(1, 2).repeat_interleave(h // hkv, 1)
            vh = qkv[..., (h + hkv) * d:].reshape(b, local, hkv, d).transpose(1, 2).repeat_interleave(h // hkv, 1)
            out = ring_attention(qh, kh, vh, cp, causal=self.causal)
            return out.transpose(1, 2).reshape(b, local, h * d).to(qkv.dtype)
        if qkv.is_cuda and not (self.dropout > 0.0 and self.training):
            from ..parallel.context_parallel import gathered_attention, gathered_attention_supported

            if gathered_attention_supported(local, d):
                return gathered_attention(qkv.contiguous(), h, hkv, d, cp, causal=self.causal).to(qkv.dtype)
        kv = gather_from_sequence_parallel_region(qkv[..., h * d:].contiguous(), cp, dim=SEQUENCE_DIM)
        b, total = q.shape[0], kv.shape[1]
        qf = q.reshape(b, local, h, d).transpose(1, 2).float()
        kf = kv[..., : hkv * d].reshape(b, total, hkv, d).transpose(1, 2).float().repeat_interleave(h // hkv, 1)
        vf = kv[..., hkv * d:].reshape(b, total, hkv, d).transpose(1, 2).float().repeat_interleave(h // hkv, 1)
        scores = qf @ kf.transpose(-1, -2) / d**0.5
        if self.causal:
            q_pos = torch.arange(offset, offset + local, device=qkv.device)[:, None]
            k_pos = torch.arange(total, device=qkv.device)[None, :]
            scores = scores.masked_fill(k_pos > q_pos, float("-inf"))
        w = torch.softmax(scores, dim=-1)
        if self.dropout > 0.0 and self.training:
            w = F.dropout(w, p=self.dropout)
        return (w @ vf).transpose(1, 2).reshape(b, local, h * d).to(qkv.dtype)


def _explicit_attention(qkv: torch.Tensor, h: int, hkv: int, d: int, causal: bool, mask: torch.Tensor | None,
                        dropout: float) -> torch.Tensor:
    """Materialised-score attention, only for additive masks or attention dropout (CPU reference semantics)."""
    if qkv.is_cuda:
        raise UnsupportedFeatureError(format_error(
            "models.attention", "explicit attention masks and attention dropout are not implemented by the flash kernel",
            expected="attention_mask=None and dropout=0 on CUDA", observed="mask or dropout given",
            resolution="are masked by causality and disable attention dropout"))
    b, s, _ = qkv.shape
    q = qkv[..., : h * d].reshape(b, s, h, d).transpose(1, 2).float()
    k = qkv[..., h * d:(h + hkv) * d].reshape(b, s, hkv, d).transpose(1, 2).float().repeat_interleave(h // hkv, 1)
    v = qkv[..., (h + hkv) * d:].reshape(b, s, hkv, d).transpose(1, 2).float().repeat_interleave(h // hkv, 1)
    scores = q @ k.transpose(-1, -2) / d**0.5
    if causal:
        scores = scores.masked_fill(torch.ones(s, s, dtype=torch.bool, device=qkv.device).triu(1), float("-inf"))
    if mask is not None:
        scores = scores + mask
    w = torch.softmax(scores, dim=-1)
    if dropout > 0:
        w = F.dropout(w, p=dropout)
    return (w @ v).transpose(1, 2).reshape(b, s, h * d).to(qkv.dtype)


class TransformerBlock(nn.Module):
    """Pre-norm block: ``x + attn(norm(x))`` then ``+ ffn(norm(.))``."""

    def __init__(self, config: ModelConfig, plan: ParallelPlan, *, layer_index: int = 0, init_seed: int = 0,
                 device: torch.device | None = None, dtype: torch.dtype | None = None,
                 compute_dtype: torch.dtype | None = None) -> None:
        super().__init__()
        seed = derive_seed(init_seed, "block", layer_index)
        self.compute_dtype = compute_dtype
        self.input_norm = _make_norm(config, plan, device, dtype)
        self.attention = TensorParallelAttention(
            config.hidden_size, config.num_heads, plan, num_kv_heads=config.resolved_num_kv_heads, dropout=config.dropout,
            bias=config.bias, causal=True, init_seed=derive_seed(seed, "attn"), device=device, dtype=dtype,
            rope_theta=config.rope_theta if config.position_embedding == "rope" else None)
        self.post_attention_norm = _make_norm(config, plan, device, dtype)
        self.feed_forward = TensorParallelFeedForward(config.hidden_size, config.resolved_ffn_hidden_size, plan.tensor_group,
                                                      activation=config.activation, bias=config.bias,
                                                      sequence_parallel=plan.sequence_parallel, init_seed=derive_seed(seed, "ffn"),
                                                      device=device, dtype=dtype)
        self.dropout = config.dropout

    def _drop(self, x: torch.Tensor) -> torch.Tensor:
        return F.dropout(x, p=self.dropout) if self.dropout > 0.0 and self.training else x

    def forward_fused(self, residual: torch.Tensor, delta: torch.Tensor | None,
                      attention_mask: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """``(residual, pending delta)`` in, ``(residual, pending delta)`` out; the adds run inside the norms."""
        if delta is None:
            h = self.input_norm(residual, out_dtype=self.compute_dtype)
        else:
            residual, h = self.input_norm(residual, delta, out_dtype=self.compute_dtype)
        a = self._drop(self.attention(h, attention_mask))
        residual, h = self.post_attention_norm(residual, a, out_dtype=self.compute_dtype)
        return residual, self._drop(self.feed_forward(h))

    def forward(self, x: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        residual, delta = self.forward_fused(x, None, attention_mask)
        return residual + delta.to(residual.dtype)


class TinyTransformer(nn.Module):
    """The decoder model; see the module docstring."""

    def __init__(self, config: ModelConfig, plan: ParallelPlan | None = None, *, seed: int = 0, device: torch.device | None = None,
                 dtype: torch.dtype | None = None, compute_dtype: torch.dtype | None = None) -> None:
        super().__init__()
        if config.kind != "transformer":
            raise ConfigurationError(format_error("models.TinyTransformer", "this class builds ModelConfig(kind='transformer') models only", expected="transformer",
                                                  observed=config.kind, resolution="use kind='transformer' in the model config"))
        self.config = config
        self.plan = plan if plan is not None else ParallelPlan.single_process()
        tp = self.plan.tensor_group
        if config.tie_word_embeddings and self.plan.vocab_parallel and tp.size > 1:
            raise UnsupportedFeatureError(format_error(
                "models.TinyTransformer", "tied embeddings with a vocabulary-parallel embedding are not supported: the "
                "embedding is split by vocabulary rows while the head needs the same matrix split by output features",
                expected="untied head weights when the vocabulary is split", observed="both enabled",
                resolution="set tie_word_embeddings=False, or keep the vocabulary whole"))
        self.compute_dtype = compute_dtype
        vocab_group = tp if self.plan.vocab_parallel else GroupHandle.trivial("tensor")
        self.token_embedding = VocabParallelEmbedding(config.vocab_size, config.hidden_size, vocab_group,
                                                      init_seed=derive_seed(seed, "token-embedding"), device=device, dtype=dtype)
        self.position_embedding: LearnedPositionEmbedding | None = None
        if config.position_embedding == "learned":
            with temporary_seed(derive_seed(seed, "position-embedding")):
                table = torch.empty(config.max_sequence_length, config.hidden_size, device=device, dtype=dtype)
                nn.init.normal_(table, mean=0.0, std=0.02)
            self.position_embedding = LearnedPositionEmbedding(config.max_sequence_length, config.hidden_size, device=device,
                                                               dtype=dtype)
            with torch.no_grad():
                self.position_embedding.weight.copy_(table)
        self.blocks = nn.ModuleList([
            TransformerBlock(config, self.plan, layer_index=i, init_seed=derive_seed(seed, "blocks"), device=device, dtype=dtype,
                             compute_dtype=compute_dtype) for i in range(config.num_layers)])
        self.final_norm = _make_norm(config, self.plan, device, dtype)
        self.output_projection = VocabParallelHead(config.hidden_size, config.vocab_size, tp, bias=False, gather_output=True,
                                                   sequence_parallel=False, init_seed=derive_seed(seed, "output-projection"),
                                                   device=device, dtype=dtype)
        if self.plan.context_parallel:
            # Every rank runs every layer on its own chunk of positions with full weights, so every
            # gradient is a partial sum over the sequence group (reduced like the SP norm weights).
            for p in self.parameters():
                p.sequence_parallel_partial_grad = True
        if config.tie_word_embeddings:
            self.output_projection.weight = self.token_embedding.weight
            # The native backward of the head and of the embedding each write into the shared
            # weight's main_grad; the weight is complete after both.
            self.token_embedding.weight.native_grad_uses = 2
        self.dropout = config.dropout

    def _embed(self, token_ids: torch.Tensor) -> torch.Tensor:
        from ..parallel.fsdp import FullyShardedDataParallel

        emb, pos = self.token_embedding, self.position_embedding
        # Sub-modules are always *called*, never read from, so an FSDP unit wrapping one of them has
        # its parameters gathered.  The position rows are fused into the gather kernel when they
        # belong to this module's own unit and the vocabulary is not split.
        if pos is not None and not isinstance(pos, FullyShardedDataParallel) and emb.group.size == 1:
            return emb(token_ids, pos.weight)
        out = emb(token_ids)
        return out if pos is None else pos(out)

    def forward(self, token_ids: torch.Tensor, attention_mask: torch.Tensor | None = None, *,
                targets: torch.Tensor | None = None) -> torch.Tensor:
        """Logits ``[B, S, V]``; or, with ``targets``, the mean next-token cross-entropy."""
        b, s = token_ids.shape
        if s > self.config.max_sequence_length:
            raise ConfigurationError(format_error("models.TinyTransformer.forward", "sequence longer than the model supports",
                                                  expected=f"<= {self.config.max_sequence_length}", observed=s,
                                                  resolution="increase max_sequence_length in the model config, or feed shorter sequences"))
        hidden = self._embed(token_ids)
        if self.dropout > 0.0 and self.training:
            hidden = F.dropout(hidden, p=self.dropout)
        info: SequenceShardInfo | None = None
        sp_group = self.plan.sequence_group
        if self.plan.sequence_parallel:
            hidden, info = pad_sequence_dimension(hidden, sp_group.size, dim=SEQUENCE_DIM)
            if attention_mask is not None and info.requires_padding:
                raise UnsupportedFeatureError(format_error(
                    "models.TinyTransformer.forward", "an explicit attention mask with sequence padding is not supported",
                    expected="a length that splits evenly over the sequence ranks",
                    observed=f"length {s}, group {sp_group.size}", resolution="pad the batch or drop the explicit mask"))
            hidden = scatter_sequence(hidden, sp_group, dim=SEQUENCE_DIM)
        residual, delta = hidden, None
        for block in self.blocks:
            residual, delta = block.forward_fused(residual, delta, attention_mask)
        if delta is None:
            h = self.final_norm(residual, out_dtype=self.compute_dtype)
        else:
            _, h = self.final_norm(residual, delta, out_dtype=self.compute_dtype)
        head = self.output_projection
        if self.plan.context_parallel:
            return self._context_parallel_head(h, targets, info)
        vocab_split = targets is not None and head.group.size > 1
        if self.plan.sequence_parallel:
            # With a vocab-split loss every rank's head produces a partial gradient for the whole
            # sequence, so the gather's adjoint must sum over ranks (reduce-scatter), not slice.
            gather = gather_from_sequence_parallel_region if vocab_split else gather_sequence
            h = gather(h, sp_group, dim=SEQUENCE_DIM)
            h = unpad_sequence_dimension(h, info, dim=SEQUENCE_DIM)
        elif vocab_split:
            h = copy_to_group(h, head.group)
        return head(h) if targets is None else head(h, targets=targets)

    def _context_parallel_head(self, h: torch.Tensor, targets: torch.Tensor | None, info: SequenceShardInfo | None) -> torch.Tensor:
        """Head and loss on the local chunk; the mean loss is summed over the sequence group."""
        cp = self.plan.sequence_group
        if targets is None:
            logits = gather_sequence(self.output_projection(h), cp, dim=SEQUENCE_DIM)
            return logits if info is None else unpad_sequence_dimension(logits, info, dim=SEQUENCE_DIM)
        if info is not None and info.requires_padding:
            raise UnsupportedFeatureError(format_error(
                "models.TinyTransformer.forward", "the loss under context parallelism needs a sequence length divisible by "
                "the sequence-parallel size", expected=f"length % {cp.size} == 0", observed=targets.shape[1],
                resolution="pad sequences so that their length splits over the sequence ranks"))
        lo, hi = local_sequence_slice(targets.shape[1], cp)
        local_mean = self.output_projection(h, targets=targets[:, lo:hi].contiguous())
        # Chunks have equal token counts: the global mean is the average of the chunk means.  The
        # reduction's adjoint passes the gradient through, so each rank backpropagates its chunk.
        return reduce_from_group(local_mean / cp.size, cp)

    def local_positions(self, sequence_length: int) -> tuple[int, int]:
        if not self.plan.sequence_parallel:
            return 0, sequence_length
        return local_sequence_slice(sequence_length, self.plan.sequence_group)

    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters())

    def __repr__(self) -> str:
        c = self.config
        sp = self.plan.sequence_group.size if self.plan.sequence_parallel else 1
        return (f"TinyTransformer(layers={c.num_layers}, hidden={c.hidden_size}, heads={c.num_heads}/{c.resolved_num_kv_heads}, "
                f"vocab={c.vocab_size}, norm={c.norm}, pos={c.position_embedding}, act={c.activation}, "
                f"tp={self.plan.tensor_group.size}, sp={sp})")


def build_reference_linear(in_features: int, out_features: int, *, bias: bool = True, init_seed: int = 0,
                           device: torch.device | None = None, dtype: torch.dtype | None = None) -> nn.Linear:
    """An ``nn.Linear`` initialised exactly like a width-1 column/row-parallel layer with the same seed."""
    linear = nn.Linear(in_features, out_features, bias=bias, device=device, dtype=dtype)
    with temporary_seed(derive_seed(init_seed, "tensor-parallel-init")), torch.no_grad():
        w = torch.empty(out_features, in_features, device=device, dtype=dtype)
        b = torch.empty(out_features, device=device, dtype=dtype) if bias else None
        init_linear_parameters(w, b, in_features=in_features)
        linear.weight.copy_(w)
        if b is not None:
            linear.bias.copy_(b)
    return linear
