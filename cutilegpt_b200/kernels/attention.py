"""Causal self-attention operators (replace cutile_gpt/kernels/attention.py:119-232)."""
from __future__ import annotations

import math

import torch

from . import ops
from ._common import as_cuda, same_dtype


def cutile_causal_attention(q, k, v, n_head: int) -> torch.Tensor:
    """softmax(q·kᵀ/√D + causal mask)·v for (batch, n_head, seq_len, head_dim) inputs.

    Any strides with a contiguous head_dim are read in place (no contiguous
    copies); the output is a new contiguous (B, H, T, D) tensor.
    """
    q, k, v = as_cuda(q, "q"), as_cuda(k, "k"), as_cuda(v, "v")
    same_dtype(q, k, v)
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("causal_attention: q, k, v must share shape (batch, n_head, seq_len, head_dim)")
    if q.shape[1] != n_head:
        raise ValueError(f"causal_attention: n_head={n_head} but q has {q.shape[1]} heads")
    q, k, v = (t if t.stride(-1) == 1 else t.contiguous() for t in (q, k, v))
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    return ops.attention_prefill(q, k, v, out, scale=1.0 / math.sqrt(q.shape[-1]))


def cutile_mha_forward(x, c_attn_weight, c_attn_bias, c_proj_weight, c_proj_bias, n_head: int,
                       c_attn_weight_t=None, c_proj_weight_t=None) -> torch.Tensor:
    """QKV projection -> causal attention -> output projection (attention.py:178-232).

    Attention reads q/k/v straight out of the fused QKV buffer and writes the
    (B, T, C) layout c_proj consumes, so no split/transpose copies happen.
    """
    x = as_cuda(x, "x")
    B, T, C = x.shape
    D = C // n_head
    x2 = x.reshape(B * T, C).contiguous()
    qkv = torch.empty((B * T, 3 * C), dtype=x.dtype, device=x.device)
    ops.gemm(x2, c_attn_weight.contiguous(), qkv, bias=c_attn_bias)
    q4 = qkv.view(B, T, 3, n_head, D)
    y = torch.empty((B, T, C), dtype=x.dtype, device=x.device)
    ops.attention_prefill(q4[:, :, 0].transpose(1, 2), q4[:, :, 1].transpose(1, 2),
                          q4[:, :, 2].transpose(1, 2), y.view(B, T, n_head, D).transpose(1, 2))
    out = torch.empty((B * T, C), dtype=x.dtype, device=x.device)
    ops.gemm(y.view(B * T, C), c_proj_weight.contiguous(), out, bias=c_proj_bias)
    return out.view(B, T, C)
