"""MLP operator (replaces cutile_gpt/kernels/fused_mlp.py:112-161).

The reference's single-kernel fusion recomputes the hidden tile per output
tile and was dropped from its model as 3-14x slower. Here the symbol maps to
two tensor-core GEMMs with fused epilogues: c_fc + bias + tanh-GELU, then
c_proj + bias. The hidden activation makes one HBM round trip.
"""
from __future__ import annotations

import torch

from .. import _lib as L
from . import ops
from ._common import as_cuda, same_dtype


def cutile_fused_mlp(x, w_fc, b_fc, w_proj, b_proj) -> torch.Tensor:
    """c_proj(gelu(c_fc(x))) over the last dimension."""
    x = as_cuda(x, "x")
    w_fc, b_fc = as_cuda(w_fc, "w_fc").contiguous(), as_cuda(b_fc, "b_fc").contiguous()
    w_proj, b_proj = as_cuda(w_proj, "w_proj").contiguous(), as_cuda(b_proj, "b_proj").contiguous()
    same_dtype(x, w_fc, b_fc, w_proj, b_proj)
    C = x.shape[-1]
    x2 = x.reshape(-1, C).contiguous()
    h = torch.empty((x2.shape[0], w_fc.shape[0]), dtype=x.dtype, device=x.device)
    ops.gemm(x2, w_fc, h, bias=b_fc, epilogue=L.EPI_BIAS_GELU)
    y = torch.empty((x2.shape[0], w_proj.shape[0]), dtype=x.dtype, device=x.device)
    ops.gemm(h, w_proj, y, bias=b_proj)
    return y.reshape(*x.shape[:-1], w_proj.shape[0])
