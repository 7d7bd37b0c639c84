"""LayerNorm operator (replaces cutile_gpt/kernels/layernorm.py:77-135).

Any normalised width is handled in place; the reference pads to a power of
two with host-side copies (layernorm.py:103-126).
"""
from __future__ import annotations

import torch

from . import ops
from ._common import as_cuda, same_dtype


def cutile_layer_norm(x, weight, bias, eps: float = 1e-5) -> torch.Tensor:
    """LayerNorm over the last dimension; same shape and dtype as x."""
    x = as_cuda(x, "x").contiguous()
    weight = as_cuda(weight, "weight").contiguous()
    bias = as_cuda(bias, "bias").contiguous()
    same_dtype(x, weight, bias)
    if weight.numel() != x.shape[-1] or bias.numel() != x.shape[-1]:
        raise ValueError(f"layer_norm: weight/bias must have {x.shape[-1]} elements")
    y = torch.empty_like(x)
    return ops.layernorm(x, weight, bias, y, eps)
