"""CPU oracle for cutileGPT's forward / generate path — TEST INFRASTRUCTURE ONLY.

This module restates the reference algorithm on the CPU with plain torch
tensor arithmetic (fp64 by default) so the CUDA path can be checked against
it. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import it, and only as the checker or the timed CPU baseline; the product
package never imports it.

Where it is pinned (tests/test_oracle.py):
  * tests/golden/reference_golden.pt — outputs of the reference's OWN code:
    cutile_gpt/models/gpt.py forward (gpt.py:95-183), generate with top_k=1
    (gpt.py:185-229, crop past block_size included) and load_from_mingpt,
    with the cutile_* kernels bound to the reference's own CuPy oracles
    (cupy_embedding / cupy_layer_norm / cupy_linear / cupy_gelu /
    cupy_causal_attention) and cupy replaced by NumPy, run in float64 by
    tests/golden/make_reference_golden.py; GPT-2 124M, nano and a crop case.
    This restatement matches them to 1e-6 (logits) and exactly (greedy ids).
  * tests/golden/golden.pt — transformers' GPT2LMHeadModel (an independent
    implementation of the same math) and torch.nn.functional per-kernel
    cases, from tests/golden/make_golden.py.
minGPT itself (third-party submodule external/minGPT, commit not visible in
the mount) is not present; the reference's tests store no values.

Every function cites the reference file:line it follows.
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import torch

SQRT_2_OVER_PI = math.sqrt(2.0 / math.pi)   # cutile_gpt/kernels/gelu.py:16
GELU_COEF = 0.044715                         # cutile_gpt/kernels/gelu.py:17


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """Two-pass mean / biased variance over the last dim (cutile_gpt/kernels/layernorm.py:139-149)."""
    mean = x.mean(dim=-1, keepdim=True)
    var = ((x - mean) ** 2).mean(dim=-1, keepdim=True)
    return w * ((x - mean) / torch.sqrt(var + eps)) + b


def gelu(x: torch.Tensor) -> torch.Tensor:
    """tanh-GELU (cutile_gpt/kernels/gelu.py:114-116)."""
    return 0.5 * x * (1.0 + torch.tanh(SQRT_2_OVER_PI * (x + GELU_COEF * x ** 3)))


def linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x · wᵀ + b with w [out, in] (cutile_gpt/kernels/linear.py:226-232)."""
    y = x @ w.t()
    return y if b is None else y + b


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """softmax(q kᵀ / √D + causal −inf mask) v on [B, H, T, D] (cutile_gpt/kernels/attention.py:236-254)."""
    T, D = q.shape[-2], q.shape[-1]
    att = (q @ k.transpose(-1, -2)) * (1.0 / math.sqrt(D))
    mask = torch.ones(T, T, dtype=torch.bool).tril()
    att = att.masked_fill(~mask, float('-inf'))
    att = torch.exp(att - att.max(dim=-1, keepdim=True).values)
    att = att / att.sum(dim=-1, keepdim=True)
    return att @ v


def embedding(idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """w[idx] (cutile_gpt/kernels/embedding.py:148-150)."""
    return w[idx]


def cast_weights(weights: Dict[str, torch.Tensor], dtype=torch.float64,
                 round_to: Optional[torch.dtype] = None) -> Dict[str, torch.Tensor]:
    """Copies a weight dict to `dtype`, optionally rounding through `round_to` first (e.g. bf16)."""
    out = {}
    cache = {}
    for k, t in weights.items():
        key = id(t)
        if key not in cache:
            u = t.detach().cpu()
            if round_to is not None:
                u = u.to(round_to)
            cache[key] = u.to(dtype)
        out[k] = cache[key]
    return out


def gpt_forward(weights: Dict[str, torch.Tensor], n_layer: int, n_head: int, idx: torch.Tensor,
                last_only: bool = False) -> torch.Tensor:
    """GPT-2 forward in the weights' dtype (cutile_gpt/models/gpt.py:95-183).

    Pre-LN blocks: x += c_proj(attn(ln_1(x))); x += mlp(ln_2(x)); logits =
    ln_f(x) · lm_headᵀ (no bias). Returns (B, T, V) logits, or (B, V) for the
    last position when last_only.
    """
    B, T = idx.shape
    C = weights['wte'].shape[1]
    D = C // n_head
    x = embedding(idx, weights['wte']) + embedding(torch.arange(T), weights['wpe']).unsqueeze(0)
    for i in range(n_layer):
        p = f'h.{i}.'
        h = layer_norm(x, weights[p + 'ln_1.weight'], weights[p + 'ln_1.bias'])
        qkv = linear(h, weights[p + 'attn.c_attn.weight'], weights[p + 'attn.c_attn.bias'])
        q, k, v = qkv.split(C, dim=2)
        q, k, v = (t.reshape(B, T, n_head, D).transpose(1, 2) for t in (q, k, v))
        y = causal_attention(q, k, v).transpose(1, 2).reshape(B, T, C)
        x = x + linear(y, weights[p + 'attn.c_proj.weight'], weights[p + 'attn.c_proj.bias'])
        h = layer_norm(x, weights[p + 'ln_2.weight'], weights[p + 'ln_2.bias'])
        h = gelu(linear(h, weights[p + 'mlp.c_fc.weight'], weights[p + 'mlp.c_fc.bias']))
        x = x + linear(h, weights[p + 'mlp.c_proj.weight'], weights[p + 'mlp.c_proj.bias'])
    if last_only:
        x = x[:, -1:, :]
    x = layer_norm(x, weights['ln_f.weight'], weights['ln_f.bias'])
    logits = linear(x, weights['lm_head.weight'])
    return logits[:, -1, :] if last_only else logits


def generate_greedy(weights: Dict[str, torch.Tensor], n_layer: int, n_head: int, block_size: int,
                    idx: torch.Tensor, max_new_tokens: int, return_margins: bool = False):
    """Greedy generation with the reference's crop semantics (cutile_gpt/models/gpt.py:204-227, top_k=1).

    Each step re-runs the forward on the last block_size tokens (positions
    restart at 0 after the crop, gpt.py:205, :111) and appends argmax of the
    last-position logits (lowest index on ties). With return_margins, also
    returns per step the gap between the top-1 and top-2 logits, used to tell
    a genuine divergence from a near-tie flipped by rounding.
    """
    margins = []
    for _ in range(max_new_tokens):
        cond = idx if idx.shape[1] <= block_size else idx[:, -block_size:]
        logits = gpt_forward(weights, n_layer, n_head, cond, last_only=True)
        top2 = torch.topk(logits, 2, dim=-1).values
        margins.append((top2[:, 0] - top2[:, 1]))
        nxt = torch.argmax(logits, dim=-1, keepdim=True)
        idx = torch.cat([idx, nxt], dim=1)
    if return_margins:
        return idx, torch.stack(margins, dim=1)
    return idx
