"""Host-side logic that needs no GPU: configs, presets, weight init and loaders, the Tile API graph."""
import math

import numpy as np
import pytest
import torch

from cutilegpt_b200 import CutileGPT, GPTConfig
from cutilegpt_b200.api import DataAnalyzer, DType, OpType, TensorSpec, TileConfig, TileOp, configure_tiles
from cutilegpt_b200.models.init import init_state, randomize_affine, weight_names


def test_presets_match_reference_values():
    # cutile_gpt/models/config.py:20-87
    expect = {'nano': (3, 3, 48, 128), 'micro': (4, 4, 128, 256), 'mini': (6, 6, 192, 256),
              'gpt2': (12, 12, 768, 1024), 'gpt2-medium': (24, 16, 1024, 1024), 'gpt2-large': (36, 20, 1280, 1024),
              'gpt2-xl': (48, 25, 1600, 1024), 'tile-small': (4, 4, 64, 128), 'tile-medium': (6, 4, 128, 256),
              'tile-large': (8, 8, 256, 512)}
    for name, (L, H, C, T) in expect.items():
        c = GPTConfig.from_name(name)
        assert (c.n_layer, c.n_head, c.n_embd, c.block_size, c.vocab_size) == (L, H, C, T, 50257)
    with pytest.raises(ValueError):
        GPTConfig.from_name("gpt5")


def test_init_distributions_and_tying():
    cfg = GPTConfig(n_layer=4, n_head=4, n_embd=256, vocab_size=5000, block_size=64)
    w = init_state(cfg, 0)
    assert set(w) == set(weight_names(cfg))
    assert w['lm_head.weight'] is w['wte']
    assert abs(w['wte'].std().item() - 0.02) < 1e-3
    proj = torch.cat([w[f'h.{i}.mlp.c_proj.weight'].flatten() for i in range(4)])
    assert abs(proj.std().item() - 0.02 / math.sqrt(8)) < 5e-4
    assert torch.all(w['h.0.ln_1.weight'] == 1) and torch.all(w['h.0.attn.c_attn.bias'] == 0)
    assert torch.equal(init_state(cfg, 0)['wte'], w['wte'])            # seeded
    randomize_affine(w, cfg, 1)
    assert w['h.0.attn.c_attn.bias'].abs().sum() > 0


def test_loaders_map_hf_and_mingpt_layouts_on_cpu():
    cfg = GPTConfig(n_layer=2, n_head=2, n_embd=32, vocab_size=97, block_size=16)
    w = init_state(cfg, 3)
    randomize_affine(w, cfg, 4)
    hf, mg = {}, {}
    for k, t in w.items():
        if k in ('wte', 'wpe'):
            hf[f'transformer.{k}.weight'] = t
            mg[f'transformer.{k}.weight'] = t
        elif k.startswith('h.'):
            conv = k.endswith('.weight') and ('attn.' in k or 'mlp.' in k)
            hf['transformer.' + k] = t.t().contiguous() if conv else t
            mg['transformer.' + k] = t
        elif k.startswith('ln_f'):
            hf['transformer.' + k] = t
            mg['transformer.' + k] = t
    hf['lm_head.weight'] = w['wte']
    mg['lm_head.weight'] = w['wte'].clone() * 2          # minGPT's head is not tied
    m = CutileGPT(cfg, device='cpu', seed=0)
    m.load_from_state_dict(hf, layout='hf')
    for k in weight_names(cfg):
        assert torch.equal(m.weights[k], w[k]), k
    assert m.weights['lm_head.weight'] is m.weights['wte']
    m.load_from_state_dict(mg, layout='mingpt')
    assert torch.equal(m.weights['lm_head.weight'], w['wte'] * 2)
    with pytest.raises(KeyError):
        m.load_state({'wte': w['wte']})


def test_tile_config_validation():
    assert configure_tiles(128, 128, 64).tile_k == 64
    with pytest.raises(ValueError):
        TileConfig(tile_m=48)


def test_tile_graph_build_and_fusion_pass():
    x = TileOp.placeholder((2, 8, 64), DType.BFLOAT16, "x")
    w1, b1 = torch.zeros(256, 64), torch.zeros(256)
    w2, b2 = torch.zeros(64, 256), torch.zeros(64)
    g = x.linear(w1, b1, out_features=256).gelu().linear(w2, b2)
    assert g.shape == (2, 8, 64)
    assert [o.op_type for o in g._ops] == [OpType.INPUT, OpType.LINEAR_BIAS, OpType.GELU, OpType.LINEAR_BIAS]
    g._optimize_graph()
    assert [o.op_type for o in g._ops] == [OpType.INPUT, OpType.LINEAR_BIAS_GELU, OpType.LINEAR_BIAS]
    assert "LINEAR_BIAS_GELU" in g.describe()
    with pytest.raises(ValueError):
        x.linear(torch.zeros(10, 63))
    assert x.reshape(-1, 64).shape == (16, 64)
    assert x.transpose().shape == (2, 64, 8)
    att = TileOp.placeholder((2, 8, 192)).attention(n_head=4)
    assert att.shape == (2, 8, 64) and att._ops[-1].params["head_dim"] == 16
    assert isinstance(x.spec, TensorSpec)


def test_data_analyzer_recommendations():
    a = DataAnalyzer()
    short = a.analyze([[1] * 100, [2] * 50])
    assert (short.recommended_tile_m, short.sample_count) == (32, 2)
    mid = a.analyze(np.ones((4, 300), dtype=np.int64))
    assert mid.recommended_tile_m == 64 and mid.source == "array"
    long = a.analyze(["x" * 1000])
    assert long.recommended_tile_m == 128 and long.max_sequence_length == 1000
