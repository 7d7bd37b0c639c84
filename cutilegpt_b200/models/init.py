"""Seeded weight initialisation with the reference's distributions.

cutile_gpt/models/gpt.py:39-81 draws every 2-D weight from N(0, 0.02), the
two residual projections (attn.c_proj, mlp.c_proj) from
N(0, 0.02/sqrt(2·n_layer)), sets biases to 0 and LayerNorm γ=1, β=0, and ties
lm_head to wte. Its RNG is CuPy's device generator, which cannot be
reproduced; here a seeded torch.Generator on the CPU draws the same
distributions so the CUDA model and the CPU oracle can share identical
weights.
"""
from __future__ import annotations

import math
from typing import Dict

import torch

from .config import GPTConfig


def weight_names(cfg: GPTConfig):
    names = ['wte', 'wpe']
    for i in range(cfg.n_layer):
        p = f'h.{i}.'
        names += [p + 'ln_1.weight', p + 'ln_1.bias', p + 'attn.c_attn.weight', p + 'attn.c_attn.bias',
                  p + 'attn.c_proj.weight', p + 'attn.c_proj.bias', p + 'ln_2.weight', p + 'ln_2.bias',
                  p + 'mlp.c_fc.weight', p + 'mlp.c_fc.bias', p + 'mlp.c_proj.weight', p + 'mlp.c_proj.bias']
    names += ['ln_f.weight', 'ln_f.bias', 'lm_head.weight']
    return names


def init_state(cfg: GPTConfig, seed: int = 0, device: str | torch.device = 'cpu') -> Dict[str, torch.Tensor]:
    """fp32 weight dict in the reference's key layout; lm_head.weight is wte (tied)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    C, L = cfg.n_embd, cfg.n_layer
    proj_std = 0.02 / math.sqrt(2 * L)

    def randn(*shape, std=0.02):
        return torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std

    w: Dict[str, torch.Tensor] = {}
    w['wte'] = randn(cfg.vocab_size, C)
    w['wpe'] = randn(cfg.block_size, C)
    for i in range(L):
        p = f'h.{i}.'
        w[p + 'ln_1.weight'] = torch.ones(C, device=device)
        w[p + 'ln_1.bias'] = torch.zeros(C, device=device)
        w[p + 'attn.c_attn.weight'] = randn(3 * C, C)
        w[p + 'attn.c_attn.bias'] = torch.zeros(3 * C, device=device)
        w[p + 'attn.c_proj.weight'] = randn(C, C, std=proj_std)
        w[p + 'attn.c_proj.bias'] = torch.zeros(C, device=device)
        w[p + 'ln_2.weight'] = torch.ones(C, device=device)
        w[p + 'ln_2.bias'] = torch.zeros(C, device=device)
        w[p + 'mlp.c_fc.weight'] = randn(4 * C, C)
        w[p + 'mlp.c_fc.bias'] = torch.zeros(4 * C, device=device)
        w[p + 'mlp.c_proj.weight'] = randn(C, 4 * C, std=proj_std)
        w[p + 'mlp.c_proj.bias'] = torch.zeros(C, device=device)
    w['ln_f.weight'] = torch.ones(C, device=device)
    w['ln_f.bias'] = torch.zeros(C, device=device)
    w['lm_head.weight'] = w['wte']
    return w


def randomize_affine(w: Dict[str, torch.Tensor], cfg: GPTConfig, seed: int = 1, std: float = 0.02) -> None:
    """Replaces the zero biases and unit LayerNorm scales with seeded random values (in place).

    The reference init leaves biases at 0 and γ at 1, which would let a kernel
    that ignores them pass parity; tests use this to exercise every term.
    """
    g = torch.Generator(device='cpu')
    g.manual_seed(seed)
    for k in list(w.keys()):
        if k.endswith('.bias'):
            w[k] = torch.randn(w[k].shape, generator=g) * std
        elif ('ln_' in k) and k.endswith('.weight'):
            w[k] = 1.0 + torch.randn(w[k].shape, generator=g) * 0.1
