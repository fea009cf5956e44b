"""Model zoo: the MLP and the GPT-2 / Llama-shaped decoder transformer."""

from .mlp import MLP, MLPBlock, build_activation
from .transformer import ParallelPlan, TensorParallelAttention, TinyTransformer, TransformerBlock, build_reference_linear

__all__ = [
    "MLP",
    "MLPBlock",
    "ParallelPlan",
    "TensorParallelAttention",
    "TinyTransformer",
    "TransformerBlock",
    "build_activation",
    "build_reference_linear",
]
