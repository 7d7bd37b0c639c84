"""Generates tests/golden/reference_golden.pt from the reference's own code.

Run from the repo root, in a container that holds the cutileGPT sources:

    python tests/golden/make_reference_golden.py --reference <path to the cutileGPT checkout>

What runs: the reference's `CutileGPT` class (cutile_gpt/models/gpt.py), with
its own `load_from_mingpt` (gpt.py:306-343), `forward` (gpt.py:95-183) and
`generate` (gpt.py:185-229), imported unmodified from the checkout. Two things
are substituted, both at the module boundary and nothing inside a function:

  * `cupy` is a NumPy namespace (`_numpy_cupy` below): every array call the
    reference makes (`asarray`, `split`, `reshape`, `transpose`, `matmul`,
    `partition`, `cumsum`, `searchsorted`, ...) has the same NumPy meaning;
    arrays are float64 so the golden values carry no float32 rounding.
  * the `cutile_*` kernel names that gpt.py imported are rebound to the
    reference's own CuPy oracles of the same ops: `cupy_embedding`
    (kernels/embedding.py:148-150), `cupy_layer_norm` (kernels/layernorm.py:139-149),
    `cupy_linear` (kernels/linear.py:226-232), `cupy_gelu` (kernels/gelu.py:114-116),
    `cupy_causal_attention` (kernels/attention.py:236-254). The cuTile kernels
    themselves need a GPU and the `tileiras` compiler, neither present here.

Greedy generation is the reference's sampling path with top_k=1
(gpt.py:207-225): the partition keeps only the maximum, the softmax is one-hot,
and the inverse-CDF draw returns the argmax whatever the random number is.

Weights: cutilegpt_b200.models.init.init_state (reference distributions,
seeded torch RNG) plus randomize_affine, handed to the reference through its
minGPT loader as a state_dict. The fixtures store the seeds, never the
weights, so the tests rebuild the same weights.

This file and the fixture are test infrastructure; nothing in the product
reads either.
"""
import argparse
import importlib
import os
import sys
import types

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from cutilegpt_b200.models.config import GPTConfig  # noqa: E402
from cutilegpt_b200.models.init import init_state, randomize_affine  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_golden.pt")

# (name, config, weight seed, batch, prompt length, greedy steps)
CASES = [
    ("nano", GPTConfig(n_layer=3, n_head=3, n_embd=48, vocab_size=50257, block_size=1024), 11, 2, 16, 8),
    ("crop", GPTConfig(n_layer=2, n_head=2, n_embd=32, vocab_size=97, block_size=8), 12, 2, 6, 12),
    ("gpt2_124m", GPTConfig(n_layer=12, n_head=12, n_embd=768, vocab_size=50257, block_size=1024), 13, 2, 16, 32),
]


def _numpy_cupy() -> types.ModuleType:
    """A `cupy` stand-in whose array functions are NumPy's (float64 everywhere)."""
    cp = types.ModuleType("cupy")
    for name in dir(np):
        if not name.startswith("__"):
            setattr(cp, name, getattr(np, name))
    rng = np.random.default_rng(0)
    rnd = types.ModuleType("cupy.random")
    rnd.randn = lambda *shape, dtype=np.float64: rng.standard_normal(shape).astype(np.float64)
    rnd.rand = lambda: np.float64(rng.random())
    cp.random = rnd
    cp.testing = np.testing
    cuda = types.ModuleType("cupy.cuda")
    cuda.get_current_stream = lambda: None
    cp.cuda = cuda
    return cp


def load_reference(path: str):
    sys.modules["cupy"] = _numpy_cupy()
    sys.path.insert(0, path)
    G = importlib.import_module("cutile_gpt.models.gpt")
    emb = importlib.import_module("cutile_gpt.kernels.embedding")
    ln = importlib.import_module("cutile_gpt.kernels.layernorm")
    lin = importlib.import_module("cutile_gpt.kernels.linear")
    gelu = importlib.import_module("cutile_gpt.kernels.gelu")
    att = importlib.import_module("cutile_gpt.kernels.attention")
    # Signature adaptors only: gpt.py passes the cached transpose as a
    # trailing argument that the CuPy oracle does not take.
    G.cutile_embedding = emb.cupy_embedding
    G.cutile_layer_norm = ln.cupy_layer_norm
    G.cutile_linear = lambda x, w, w_t=None: lin.cupy_linear(x, w)
    G.cutile_linear_bias = lambda x, w, b, w_t=None: lin.cupy_linear(x, w, b)
    G.cutile_gelu = gelu.cupy_gelu
    G.cutile_causal_attention = att.cupy_causal_attention
    return G


class _StateDictHolder:
    """What the reference's load_from_mingpt reads: an object with state_dict()."""

    def __init__(self, sd):
        self._sd = sd

    def state_dict(self):
        return self._sd


def _mingpt_state_dict(w, cfg):
    sd = {"transformer.wte.weight": w["wte"], "transformer.wpe.weight": w["wpe"],
          "transformer.ln_f.weight": w["ln_f.weight"], "transformer.ln_f.bias": w["ln_f.bias"],
          "lm_head.weight": w["wte"]}
    for i in range(cfg.n_layer):
        for n in ("ln_1.weight", "ln_1.bias", "attn.c_attn.weight", "attn.c_attn.bias", "attn.c_proj.weight",
                  "attn.c_proj.bias", "ln_2.weight", "ln_2.bias", "mlp.c_fc.weight", "mlp.c_fc.bias",
                  "mlp.c_proj.weight", "mlp.c_proj.bias"):
            sd[f"transformer.h.{i}.{n}"] = w[f"h.{i}.{n}"]
    return {k: v.double() for k, v in sd.items()}


def run_case(G, name, cfg, seed, B, T, steps):
    w = init_state(cfg, seed)
    randomize_affine(w, cfg, seed + 100)
    model = G.CutileGPT.__new__(G.CutileGPT)      # skip the CuPy-RNG init; weights come from the loader
    model.config = G.GPTConfig(n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd,
                               vocab_size=cfg.vocab_size, block_size=cfg.block_size)
    model.weights, model.weight_transposes = {}, {}
    model.load_from_mingpt(_StateDictHolder(_mingpt_state_dict(w, cfg)))

    g = torch.Generator().manual_seed(seed + 7)
    idx = torch.randint(0, cfg.vocab_size, (B, T), generator=g)
    logits, _ = model.forward(idx.numpy())
    logits = torch.from_numpy(np.ascontiguousarray(logits))            # (B, T, V) float64

    # Record the top-1/top-2 margin of every step's last-position logits.
    margins = []
    fwd = model.forward

    def recording_forward(ids):
        out, none = fwd(ids)
        top2 = np.sort(out[:, -1, :], axis=-1)[:, -2:]
        margins.append(top2[:, 1] - top2[:, 0])
        return out, none

    model.forward = recording_forward
    seq = model.generate(idx.numpy().copy(), steps, temperature=1.0, top_k=1)
    keep = min(cfg.vocab_size, 1024)
    return {
        "config": dict(n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd, vocab_size=cfg.vocab_size,
                       block_size=cfg.block_size),
        "weight_seed": seed, "affine_seed": seed + 100, "idx": idx,
        "logits_head": logits[..., :keep].float(),
        "logits_last": logits[:, -1].float() if cfg.vocab_size <= 2048 or name == "gpt2_124m" else None,
        "logits_sum": logits.sum(-1), "logits_sqsum": (logits ** 2).sum(-1),
        "argmax": logits.argmax(-1),
        "greedy": torch.from_numpy(np.asarray(seq)).long(), "greedy_steps": steps,
        "greedy_margins": torch.from_numpy(np.stack(margins, axis=1)),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the cutileGPT source checkout")
    args = ap.parse_args()
    G = load_reference(args.reference)
    data = {"source": "cutile_gpt/models/gpt.py forward/generate with the cupy_* oracles, NumPy float64",
            "cases": {}}
    for name, cfg, seed, B, T, steps in CASES:
        data["cases"][name] = run_case(G, name, cfg, seed, B, T, steps)
        m = data["cases"][name]["greedy_margins"]
        print(f"{name}: greedy {tuple(data['cases'][name]['greedy'].shape)}, min margin {m.min().item():.3e}",
              flush=True)
    torch.save(data, OUT)
    print(f"wrote {OUT} ({os.path.getsize(OUT) / 1e6:.2f} MB)")


if __name__ == "__main__":
    main()
