"""Linear operators (replace cutile_gpt/kernels/linear.py:112-222).

``weight`` is the nn.Linear [out_features, in_features] matrix. The
bf16 path runs on the tcgen05 tensor-core GEMM, which consumes that
layout directly; ``weight_t`` (the reference's pre-transposed copy) is
accepted for signature compatibility and not needed.
"""
from __future__ import annotations

import torch

from . import ops
from ._common import as_cuda, same_dtype


def _linear(x, weight, bias) -> torch.Tensor:
    x = as_cuda(x, "x")
    weight = as_cuda(weight, "weight").contiguous()
    if bias is not None:
        bias = as_cuda(bias, "bias").contiguous()
    same_dtype(x, weight, bias)
    in_f = x.shape[-1]
    if weight.shape[1] != in_f:
        raise ValueError(f"linear: weight in_features {weight.shape[1]} != input dim {in_f}")
    x2 = x.reshape(-1, in_f)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    out = torch.empty((x2.shape[0], weight.shape[0]), dtype=x.dtype, device=x.device)
    ops.gemm(x2, weight, out, bias=bias)
    return out.reshape(*x.shape[:-1], weight.shape[0])


def cutile_linear(x, weight, weight_t=None) -> torch.Tensor:
    """y = x · weightᵀ; output dtype = x.dtype."""
    return _linear(x, weight, None)


def cutile_linear_bias(x, weight, bias, weight_t=None) -> torch.Tensor:
    """y = x · weightᵀ + bias (bias fused into the GEMM epilogue)."""
    return _linear(x, weight, bias)
