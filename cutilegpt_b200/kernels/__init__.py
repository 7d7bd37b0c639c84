"""sm_100a kernels behind the reference operator surface (cutile_gpt/kernels/__init__.py:9-24)."""
from .gelu import cutile_gelu
from .embedding import cutile_embedding, cutile_token_pos_embedding
from .linear import cutile_linear, cutile_linear_bias
from .layernorm import cutile_layer_norm
from .attention import cutile_causal_attention, cutile_mha_forward
from .fused_mlp import cutile_fused_mlp

__all__ = [
    'cutile_gelu',
    'cutile_embedding',
    'cutile_linear',
    'cutile_linear_bias',
    'cutile_layer_norm',
    'cutile_causal_attention',
    'cutile_fused_mlp',
]
