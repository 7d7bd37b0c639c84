"""cutilegpt_b200 — B200-native (sm_100a) drop-in for cutileGPT's forward path.

Mirrors the reference package facade (cutile_gpt/__init__.py:41-129): the
seven kernel operators, the model (CutileGPT, GPTConfig) and the Tile API,
with hand-written CUDA kernels behind a C ABI (include/gpt_b200.h,
libgpt_b200.so) instead of cuTile.
"""
__version__ = "0.1.0"

from .kernels import (
    cutile_gelu,
    cutile_embedding,
    cutile_linear,
    cutile_linear_bias,
    cutile_layer_norm,
    cutile_causal_attention,
    cutile_fused_mlp,
)
from .api import (
    TileOp,
    TileConfig,
    TensorSpec,
    Layout,
    DType,
    tile,
    configure_tiles,
    DataProfile,
    DataAnalyzer,
)
from .models import CutileGPT, GPTConfig

__all__ = [
    '__version__',
    'CutileGPT',
    'GPTConfig',
    'TileOp',
    'TileConfig',
    'TensorSpec',
    'Layout',
    'DType',
    'tile',
    'configure_tiles',
    'DataProfile',
    'DataAnalyzer',
    'cutile_gelu',
    'cutile_embedding',
    'cutile_linear',
    'cutile_linear_bias',
    'cutile_layer_norm',
    'cutile_causal_attention',
    'cutile_fused_mlp',
]
