"""The CPU oracle against the golden fixtures (transformers GPT2LMHeadModel and
torch.nn.functional, float64) — pins the checker before it checks anything."""
import pytest
import torch

from oracle import ref_gpt as R
from cutilegpt_b200.models.config import GPTConfig
from cutilegpt_b200.models.init import init_state, randomize_affine


def test_kernels_vs_golden(golden):
    k = golden["kernels"]
    d = lambda t: t.double()  # noqa: E731
    c = k["layernorm"]
    torch.testing.assert_close(R.layer_norm(d(c["x"]), d(c["w"]), d(c["b"])), d(c["y"]), atol=1e-6, rtol=1e-6)
    for nm in ("gelu_1d", "gelu_2d", "gelu_3d"):
        torch.testing.assert_close(R.gelu(d(k[nm]["x"])), d(k[nm]["y"]), atol=1e-6, rtol=1e-6)
    c = k["linear"]
    torch.testing.assert_close(R.linear(d(c["x"]), d(c["w"])), d(c["y"]), atol=1e-5, rtol=1e-6)
    torch.testing.assert_close(R.linear(d(c["x"]), d(c["w"]), d(c["b"])), d(c["y_bias"]), atol=1e-5, rtol=1e-6)
    c = k["attention"]
    torch.testing.assert_close(R.causal_attention(d(c["q"]), d(c["k"]), d(c["v"])), d(c["y"]),
                               atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("name", ["nano", "odd_heads"])
def test_model_vs_golden(golden, name):
    c = golden["models"][name]
    cfg = GPTConfig(**c["config"])
    w = init_state(cfg, c["weight_seed"])
    randomize_affine(w, cfg, c["affine_seed"])
    wd = R.cast_weights(w)
    logits = R.gpt_forward(wd, cfg.n_layer, cfg.n_head, c["idx"])
    keep = c["logits_head"].shape[-1]
    assert (logits[..., :keep] - c["logits_head"].double()).abs().max() < 1e-6
    torch.testing.assert_close(logits.sum(-1), c["logits_sum"], atol=1e-8, rtol=1e-10)
    torch.testing.assert_close((logits ** 2).sum(-1), c["logits_sqsum"], atol=1e-8, rtol=1e-10)
    assert torch.equal(logits.argmax(-1), c["argmax"])
    seq = R.generate_greedy(wd, cfg.n_layer, cfg.n_head, cfg.block_size, c["idx"], c["greedy_steps"])
    assert torch.equal(seq, c["greedy"])


def test_last_only_matches_full():
    cfg = GPTConfig(n_layer=2, n_head=2, n_embd=32, vocab_size=97, block_size=32)
    w = R.cast_weights(init_state(cfg, 3))
    idx = torch.randint(0, 97, (3, 9), generator=torch.Generator().manual_seed(0))
    full = R.gpt_forward(w, 2, 2, idx)
    last = R.gpt_forward(w, 2, 2, idx, last_only=True)
    torch.testing.assert_close(full[:, -1], last)


def test_greedy_crop_semantics():
    """Past block_size the prefix is cropped and positions restart at 0 (cutile_gpt/models/gpt.py:205)."""
    cfg = GPTConfig(n_layer=1, n_head=2, n_embd=16, vocab_size=50, block_size=8)
    w = R.cast_weights(init_state(cfg, 4))
    idx = torch.randint(0, 50, (2, 6), generator=torch.Generator().manual_seed(1))
    seq, margins = R.generate_greedy(w, 1, 2, 8, idx, 5, return_margins=True)
    assert seq.shape == (2, 11) and margins.shape == (2, 5)
    # the last step must equal argmax over a forward of the last 8 tokens only
    last = R.gpt_forward(w, 1, 2, seq[:, -9:-1], last_only=True).argmax(-1)
    assert torch.equal(last, seq[:, -1])


def _ref_case_weights(c):
    cfg = GPTConfig(**c["config"])
    w = init_state(cfg, c["weight_seed"])
    randomize_affine(w, cfg, c["affine_seed"])
    return cfg, R.cast_weights(w)


@pytest.mark.parametrize("name", ["nano", "crop", "gpt2_124m"])
def test_oracle_vs_reference_code(ref_golden, name):
    """The restatement against the reference's own forward/generate run under a NumPy cupy (float64)."""
    c = ref_golden["cases"][name]
    cfg, wd = _ref_case_weights(c)
    logits = R.gpt_forward(wd, cfg.n_layer, cfg.n_head, c["idx"])
    keep = c["logits_head"].shape[-1]
    assert (logits[..., :keep] - c["logits_head"].double()).abs().max() < 1e-6
    torch.testing.assert_close(logits.sum(-1), c["logits_sum"], atol=1e-8, rtol=1e-10)
    torch.testing.assert_close((logits ** 2).sum(-1), c["logits_sqsum"], atol=1e-8, rtol=1e-10)
    assert torch.equal(logits.argmax(-1), c["argmax"])
    if c["logits_last"] is not None:
        assert (logits[:, -1] - c["logits_last"].double()).abs().max() < 1e-6
    seq, margins = R.generate_greedy(wd, cfg.n_layer, cfg.n_head, cfg.block_size, c["idx"], c["greedy_steps"],
                                     return_margins=True)
    assert torch.equal(seq, c["greedy"])
    torch.testing.assert_close(margins, c["greedy_margins"], atol=1e-9, rtol=1e-7)
