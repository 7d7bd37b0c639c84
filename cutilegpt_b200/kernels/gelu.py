"""tanh-GELU operator (replaces cutile_gpt/kernels/gelu.py:71-110)."""
from __future__ import annotations

import torch

from . import ops
from ._common import as_cuda


def cutile_gelu(x) -> torch.Tensor:
    """0.5·x·(1 + tanh(√(2/π)(x + 0.044715x³))) elementwise, any shape; returns a new tensor."""
    x = as_cuda(x, "x").contiguous()
    y = torch.empty_like(x)
    return ops.gelu(x, y)
