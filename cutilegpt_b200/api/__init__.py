"""Tile API (mirrors cutile_gpt/api/__init__.py)."""
from .config import TileConfig, TensorSpec, Layout, DType, configure_tiles
from .tile_op import TileOp, OpType, OpNode, tile
from .profiler import DataProfile, DataAnalyzer

__all__ = ['TileConfig', 'TensorSpec', 'Layout', 'DType', 'configure_tiles', 'TileOp', 'OpType', 'OpNode',
           'tile', 'DataProfile', 'DataAnalyzer']
