"""Generates tests/golden/golden.pt — fixtures that pin the CPU oracle.

Run from the repo root:  python tests/golden/make_golden.py

Sources (independent implementations of the reference math, run here on
the CPU in float64):
  * transformers.GPT2LMHeadModel (activation gelu_new = tanh-GELU, LN eps
    1e-5, Conv1D weights = transposed nn.Linear, tied lm_head) with the
    seeded weights of cutilegpt_b200.models.init (reference init
    distributions, cutile_gpt/models/gpt.py:39-81) plus seeded random
    biases / LN affine so every term is exercised;
  * torch.nn.functional layer_norm / gelu(approximate='tanh') / linear /
    scaled_dot_product_attention(is_causal=True) for the per-kernel cases,
    at the shapes of the reference kernels' self-tests
    (cutile_gpt/kernels/layernorm.py:152-172, gelu.py:119-149,
    linear.py:235-263, attention.py:257-277).
The reference package itself cannot run in this container (it imports cupy,
which is not installed), and its tests store no values.
"""
import os
import sys

import torch
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from cutilegpt_b200.models.config import GPTConfig  # noqa: E402
from cutilegpt_b200.models.init import init_state, randomize_affine  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.pt")

# (name, config, weight seed, batch, seq, greedy steps)
MODEL_CASES = [
    ("nano", GPTConfig(n_layer=3, n_head=3, n_embd=48, vocab_size=50257, block_size=1024), 0, 2, 16, 8),
    ("odd_heads", GPTConfig(n_layer=2, n_head=5, n_embd=80, vocab_size=1000, block_size=24), 5, 2, 12, 16),
]


def hf_model(cfg: GPTConfig, w):
    from transformers import GPT2Config, GPT2LMHeadModel
    hc = GPT2Config(vocab_size=cfg.vocab_size, n_positions=cfg.block_size, n_embd=cfg.n_embd,
                    n_layer=cfg.n_layer, n_head=cfg.n_head, activation_function="gelu_new",
                    resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0, layer_norm_epsilon=1e-5,
                    tie_word_embeddings=True)
    m = GPT2LMHeadModel(hc).double().eval()
    sd = {}
    sd["transformer.wte.weight"] = w["wte"]
    sd["transformer.wpe.weight"] = w["wpe"]
    for i in range(cfg.n_layer):
        p, s = f"h.{i}.", f"transformer.h.{i}."
        for n in ("ln_1.weight", "ln_1.bias", "ln_2.weight", "ln_2.bias", "attn.c_attn.bias",
                  "attn.c_proj.bias", "mlp.c_fc.bias", "mlp.c_proj.bias"):
            sd[s + n] = w[p + n]
        for n in ("attn.c_attn.weight", "attn.c_proj.weight", "mlp.c_fc.weight", "mlp.c_proj.weight"):
            sd[s + n] = w[p + n].t().contiguous()   # Conv1D stores [in, out]
    sd["transformer.ln_f.weight"] = w["ln_f.weight"]
    sd["transformer.ln_f.bias"] = w["ln_f.bias"]
    sd["lm_head.weight"] = w["wte"]
    sd = {k: v.double() for k, v in sd.items()}
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all(k.endswith("attn.bias") or k.endswith("masked_bias") for k in missing), missing
    return m


def model_case(name, cfg, seed, B, T, steps):
    w = init_state(cfg, seed)
    randomize_affine(w, cfg, seed + 100)
    m = hf_model(cfg, w)
    g = torch.Generator().manual_seed(seed + 7)
    idx = torch.randint(0, cfg.vocab_size, (B, T), generator=g)
    with torch.no_grad():
        logits = m(idx).logits                          # (B, T, V) float64
        seq = idx.clone()
        for _ in range(steps):                          # greedy, crop to block_size
            cond = seq if seq.shape[1] <= cfg.block_size else seq[:, -cfg.block_size:]
            nxt = m(cond).logits[:, -1].argmax(-1, keepdim=True)
            seq = torch.cat([seq, nxt], 1)
    V = cfg.vocab_size
    keep = min(V, 1024)
    return {
        "config": dict(n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd, vocab_size=V,
                       block_size=cfg.block_size),
        "weight_seed": seed, "affine_seed": seed + 100, "idx": idx,
        "logits_head": logits[..., :keep].float(),     # first `keep` vocab entries, all positions
        "logits_sum": logits.sum(-1), "logits_sqsum": (logits ** 2).sum(-1),
        "argmax": logits.argmax(-1), "greedy": seq, "greedy_steps": steps,
    }


def kernel_cases():
    g = torch.Generator().manual_seed(1234)
    rn = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    out = {}
    out["layernorm"] = _fp32_case(dict(x=rn(2, 64, 48), w=rn(48), b=rn(48)),
                                  lambda d: dict(y=F.layer_norm(d["x"], (48,), d["w"], d["b"], eps=1e-5)))
    for nm, shp in (("gelu_1d", (1024,)), ("gelu_2d", (128, 256)), ("gelu_3d", (2, 64, 48))):
        out[nm] = _fp32_case(dict(x=rn(*shp)), lambda d: dict(y=F.gelu(d["x"], approximate="tanh")))
    out["linear"] = _fp32_case(dict(x=rn(2, 64, 48), w=rn(192, 48), b=rn(192)),
                               lambda d: dict(y=F.linear(d["x"], d["w"]),
                                              y_bias=F.linear(d["x"], d["w"], d["b"])))
    out["attention"] = _fp32_case(
        dict(q=rn(2, 3, 32, 16), k=rn(2, 3, 32, 16), v=rn(2, 3, 32, 16)),
        lambda d: dict(y=F.scaled_dot_product_attention(d["q"], d["k"], d["v"], is_causal=True)))
    # Inputs are rounded to fp32 before the fp64 reference is computed, so
    # the stored fp32 inputs reproduce it; outputs are stored as fp32.
    return out


def _fp32_case(fn_inputs, make):
    ins = {k: v.float().double() for k, v in fn_inputs.items()}
    outs = make(ins)
    return {**{k: v.float() for k, v in ins.items()}, **{k: v.float() for k, v in outs.items()}}


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    data = {"models": {n: model_case(n, c, s, B, T, st) for n, c, s, B, T, st in MODEL_CASES},
            "kernels": kernel_cases(), "torch": torch.__version__}
    torch.save(data, OUT)
    print(f"wrote {OUT} ({os.path.getsize(OUT) / 1e6:.2f} MB)")


if __name__ == "__main__":
    main()
