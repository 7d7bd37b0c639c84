"""Embedding gather (replaces cutile_gpt/kernels/embedding.py:54-144).

No padding copies: the reference pads the whole weight to a power-of-two
width on every call (embedding.py:77-82); here rows are gathered directly.
"""
from __future__ import annotations

import torch

from . import ops
from ._common import as_cuda


def cutile_embedding(indices, weight) -> torch.Tensor:
    """weight[indices] with shape (*indices.shape, n_embd) in weight's dtype."""
    indices = as_cuda(indices, "indices")
    weight = as_cuda(weight, "weight").contiguous()
    idx = indices.to(torch.int64).contiguous()
    out = torch.empty((*indices.shape, weight.shape[1]), dtype=weight.dtype, device=weight.device)
    return ops.embedding(idx, weight, out)


def cutile_token_pos_embedding(token_ids, token_weight, pos_weight, input_pos: int = 0) -> torch.Tensor:
    """token_weight[token_ids] + pos_weight[input_pos + t] in one pass (embedding.py:112-144)."""
    token_ids = as_cuda(token_ids, "token_ids")
    wte = as_cuda(token_weight, "token_weight").contiguous()
    wpe = as_cuda(pos_weight, "pos_weight").contiguous()
    ids = token_ids.to(torch.int64).contiguous()
    if ids.dim() == 1:
        ids = ids.unsqueeze(0)
    out = torch.empty((*ids.shape, wte.shape[1]), dtype=wte.dtype, device=wte.device)
    ops.embedding_pos(ids, wte, wpe, out, pos0=input_pos)
    return out.reshape(*token_ids.shape, wte.shape[1])
