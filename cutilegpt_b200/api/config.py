"""Tile API configuration types (same names and fields as cutile_gpt/api/config.py:12-120).

Tile sizes here are advisory, as in the reference (its kernels never read
them): the sm_100a kernels pick their own tiles (BN in gemm_tc.cu, split
counts in gemm_skinny.cu / decode.cu).
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import Enum, auto
from typing import Tuple

import torch


class Layout(Enum):
    ROW_MAJOR = auto()
    COL_MAJOR = auto()
    TILED = auto()


class DType(Enum):
    FLOAT32 = auto()
    FLOAT16 = auto()
    BFLOAT16 = auto()

    def to_torch(self) -> torch.dtype:
        return {DType.FLOAT32: torch.float32, DType.FLOAT16: torch.float16,
                DType.BFLOAT16: torch.bfloat16}[self]

    def to_cupy(self):
        import cupy as cp  # optional dependency, as in the reference
        return {DType.FLOAT32: cp.float32, DType.FLOAT16: cp.float16,
                DType.BFLOAT16: cp.dtype('bfloat16')}[self]

    @staticmethod
    def from_torch(dt: torch.dtype) -> 'DType':
        return {torch.float32: DType.FLOAT32, torch.float16: DType.FLOAT16,
                torch.bfloat16: DType.BFLOAT16}.get(dt, DType.FLOAT32)


@dataclass
class TileConfig:
    """Explicit tile configuration; sizes must be powers of two (reference: config.py:37-65)."""
    tile_m: int = 64
    tile_n: int = 64
    tile_k: int = 32
    num_ctas: int = 1
    occupancy: int = 4
    latency_hint: int = 4
    use_tma: bool = True
    use_swizzle: bool = True
    use_tf32: bool = True

    def __post_init__(self):
        for name in ('tile_m', 'tile_n', 'tile_k'):
            v = getattr(self, name)
            if v <= 0 or (v & (v - 1)) != 0:
                raise ValueError(f"{name}={v} must be power of 2")


@dataclass
class TensorSpec:
    """Shape / dtype / layout / name of a tensor in a Tile graph."""
    shape: Tuple[int, ...]
    dtype: DType = DType.FLOAT32
    layout: Layout = Layout.ROW_MAJOR
    name: str = ""
    dim_names: Tuple[str, ...] = ()

    @property
    def ndim(self) -> int:
        return len(self.shape)

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    def with_shape(self, *shape) -> 'TensorSpec':
        return TensorSpec(shape=shape, dtype=self.dtype, layout=self.layout, name=self.name,
                          dim_names=self.dim_names)

    def __repr__(self) -> str:
        dims = f", dims={self.dim_names}" if self.dim_names else ""
        return f"TensorSpec({self.name}: {self.shape}, {self.dtype.name}, {self.layout.name}{dims})"


def configure_tiles(tile_m: int = 64, tile_n: int = 64, tile_k: int = 32, **kwargs) -> TileConfig:
    return TileConfig(tile_m=tile_m, tile_n=tile_n, tile_k=tile_k, **kwargs)
