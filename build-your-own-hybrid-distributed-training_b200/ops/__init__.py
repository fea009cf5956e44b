"""Hand-written sm_100a kernels and the autograd ops built on them.

Every function accepts CPU tensors (plain PyTorch, used by the Gloo tests and
as the numerical oracle) and CUDA tensors (the native kernels in
``ops/csrc``; no PyTorch fallback -- a missing extension raises
:class:`~hybrid_training.errors.KernelError`).
"""

from ._ext import build_checked_extension, build_extension, checked_extension, extension, extension_path, has_extension
from .attention import apply_rope, attention, reference_attention, rope_tables
from .embedding import embedding
from .grads import deliver_grad, has_main_grad, reset_main_grad_state
from .linear import (EPI_GELU, EPI_GELU_BWD, EPI_PLAIN, compute_weight, gelu_backward, gelu_mlp, gemm, linear, reference_gemm,
                     set_deterministic_reductions, swiglu, swiglu_gemm, swiglu_mlp, swiglu_mlp_supported)
from .loss import cross_entropy, lm_head_cross_entropy, reference_vocab_parallel_cross_entropy
from .norm import add_norm, layer_norm, rms_norm
from .optim import HYPER_SLOTS, adamw_flat, grad_sumsq, reference_adamw

__all__ = [
    "EPI_GELU",
    "EPI_GELU_BWD",
    "EPI_PLAIN",
    "HYPER_SLOTS",
    "adamw_flat",
    "add_norm",
    "apply_rope",
    "attention",
    "build_checked_extension",
    "build_extension",
    "checked_extension",
    "compute_weight",
    "cross_entropy",
    "deliver_grad",
    "embedding",
    "extension",
    "extension_path",
    "gelu_backward",
    "gemm",
    "grad_sumsq",
    "has_extension",
    "has_main_grad",
    "layer_norm",
    "gelu_mlp",
    "linear",
    "lm_head_cross_entropy",
    "reference_adamw",
    "reference_attention",
    "reference_gemm",
    "reference_vocab_parallel_cross_entropy",
    "reset_main_grad_state",
    "rms_norm",
    "rope_tables",
    "set_deterministic_reductions",
    "swiglu",
    "swiglu_gemm",
    "swiglu_mlp",
    "swiglu_mlp_supported",
]
