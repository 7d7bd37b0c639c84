"""Per-kernel parity of libgpt_b200 against the fp64 CPU oracle and the golden fixtures.

Tolerances: fp32 kernels follow the reference self-tests (layernorm / linear
1e-4, gelu 1e-5, attention 1e-3: cutile_gpt/kernels/*.py __main__ blocks);
bf16 kernels are compared with the oracle run on the same bf16-rounded
inputs, within a relative error of 2e-2 (max|Δ| / max|ref|).
"""
import math

import pytest
import torch

from oracle import ref_gpt as R
from cutilegpt_b200 import _lib as L
from cutilegpt_b200.kernels import ops
import cutilegpt_b200 as cg

pytestmark = pytest.mark.gpu
BF16_REL = 2e-2


def rel_err(got, ref):
    got, ref = got.double().cpu(), ref.double().cpu()
    return ((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()


def randn(*shape, seed=0, dtype=torch.float32, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g, dtype=torch.float64) * scale).to(dtype)


def cuda(t):
    return t.cuda()


# ----------------------------------------------------------------- golden cases
def test_golden_layernorm_fp32(golden):
    c = golden["kernels"]["layernorm"]
    y = cg.cutile_layer_norm(cuda(c["x"]), cuda(c["w"]), cuda(c["b"]))
    torch.testing.assert_close(y.cpu(), c["y"], atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("name", ["gelu_1d", "gelu_2d", "gelu_3d"])
def test_golden_gelu_fp32(golden, name):
    c = golden["kernels"][name]
    y = cg.cutile_gelu(cuda(c["x"]))
    torch.testing.assert_close(y.cpu(), c["y"], atol=1e-5, rtol=1e-5)


def test_golden_linear_fp32(golden):
    c = golden["kernels"]["linear"]
    y = cg.cutile_linear(cuda(c["x"]), cuda(c["w"]))
    yb = cg.cutile_linear_bias(cuda(c["x"]), cuda(c["w"]), cuda(c["b"]))
    torch.testing.assert_close(y.cpu(), c["y"], atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(yb.cpu(), c["y_bias"], atol=1e-4, rtol=1e-4)


def test_golden_attention_fp32(golden):
    c = golden["kernels"]["attention"]
    y = cg.cutile_causal_attention(cuda(c["q"]), cuda(c["k"]), cuda(c["v"]), 3)
    torch.testing.assert_close(y.cpu(), c["y"], atol=1e-3, rtol=1e-3)


# ----------------------------------------------------------------- layernorm
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,C", [(1, 48), (130, 48), (257, 384), (64, 768), (33, 1600), (5, 100), (3, 8200)])
def test_layernorm(dtype, M, C):
    x = randn(M, C, seed=1, scale=3.0) + 0.5
    w, b = randn(C, seed=2) * 0.1 + 1.0, randn(C, seed=3) * 0.1
    xd, wd, bd = (t.to(dtype) for t in (x, w, b))
    y = cg.cutile_layer_norm(cuda(xd), cuda(wd), cuda(bd))
    ref = R.layer_norm(xd.double(), wd.double(), bd.double())
    if dtype == torch.float32:
        torch.testing.assert_close(y.cpu().double(), ref, atol=1e-4, rtol=1e-4)
    else:
        assert rel_err(y, ref) < BF16_REL


# ----------------------------------------------------------------- gelu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [1, 7, 1024, 12345, 32 * 512 * 768])
def test_gelu(dtype, n):
    x = randn(n, seed=4, scale=3.0).to(dtype)
    y = cg.cutile_gelu(cuda(x))
    ref = R.gelu(x.double())
    if dtype == torch.float32:
        torch.testing.assert_close(y.cpu().double(), ref, atol=1e-5, rtol=1e-5)
    else:
        # bf16 output rounding (2^-9 relative) dominates
        torch.testing.assert_close(y.cpu().double(), ref, atol=1e-2, rtol=8e-3)


def test_gelu_unaligned_view():
    x = randn(1001, seed=5).cuda()
    y = torch.empty_like(x)
    ops.gelu(x[1:], y[1:])
    torch.testing.assert_close(y[1:].cpu().double(), R.gelu(x[1:].cpu().double()), atol=1e-5, rtol=1e-5)


# ----------------------------------------------------------------- embedding
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("C", [48, 768, 1600, 100])
def test_embedding(dtype, C):
    V, B, T = 1000, 3, 37
    wte, wpe = randn(V, C, seed=6).to(dtype), randn(64, C, seed=7).to(dtype)
    idx = torch.randint(0, V, (B, T), generator=torch.Generator().manual_seed(8))
    e = cg.cutile_embedding(idx.cuda(), wte.cuda())
    assert e.shape == (B, T, C)
    assert torch.equal(e.cpu(), wte[idx])
    out = torch.empty((B, T, C), dtype=dtype, device="cuda")
    ops.embedding_pos(idx.cuda(), wte.cuda(), wpe.cuda(), out, pos0=5)
    ref = (wte.double()[idx] + wpe.double()[5:5 + T].unsqueeze(0)).to(dtype)
    assert torch.equal(out.cpu(), ref)


def test_embedding_out_of_range_reports():
    w = randn(10, 16, seed=9).cuda()
    idx = torch.tensor([[1, 12]], device="cuda")
    out = cg.cutile_embedding(idx, w)
    with pytest.raises(L.GptError):
        L.device_error()
    assert torch.all(out[0, 1] == 0)
    assert L.device_error() == 0  # cleared


# ----------------------------------------------------------------- gemm
EPIS = [L.EPI_NONE, L.EPI_BIAS, L.EPI_BIAS_GELU, L.EPI_BIAS_RESIDUAL]


def gemm_ref(a, w, bias, r, epi):
    y = a.double() @ w.double().t()
    if epi != L.EPI_NONE:
        y = y + bias.double()
    if epi == L.EPI_BIAS_GELU:
        y = R.gelu(y)
    if epi == L.EPI_BIAS_RESIDUAL:
        y = y + r.double()
    return y


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("epi", EPIS)
@pytest.mark.parametrize("M,N,K", [(64, 192, 48), (128, 256, 64), (200, 2304, 768), (300, 768, 3072),
                                   (129, 50257, 48), (64, 3072, 768), (8, 768, 768), (1000, 129, 1600),
                                   (513, 2304, 768), (1000, 50257, 64), (2048, 768, 3072)])
def test_gemm(dtype, epi, M, N, K):
    a = randn(M, K, seed=10).to(dtype)
    w = (randn(N, K, seed=11) / math.sqrt(K)).to(dtype)
    bias = randn(N, seed=12).to(dtype)
    r = randn(M, N, seed=13).to(dtype)
    out = torch.empty((M, N), dtype=dtype, device="cuda")
    ops.gemm(a.cuda(), w.cuda(), out, bias=bias.cuda(), resid=r.cuda() if epi == L.EPI_BIAS_RESIDUAL else None,
             epilogue=epi)
    ref = gemm_ref(a, w, bias, r, epi)
    if dtype == torch.float32:
        torch.testing.assert_close(out.cpu().double(), ref, atol=1e-4, rtol=1e-4)
    else:
        assert rel_err(out, ref) < BF16_REL, rel_err(out, ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gemm_strided_and_inplace_residual(dtype):
    M, N, K = 96, 384, 384
    big = randn(M, 2 * K, seed=14).to(dtype).cuda()
    a = big[:, 8:8 + K]                        # row stride 2K, 16-byte aligned offset
    w = (randn(N, K, seed=15) / math.sqrt(K)).to(dtype).cuda()
    bias = randn(N, seed=16).to(dtype).cuda()
    x = randn(M, N, seed=17).to(dtype).cuda()
    ref = gemm_ref(a.cpu(), w.cpu(), bias.cpu(), x.cpu(), L.EPI_BIAS_RESIDUAL)
    ops.gemm(a, w, x, bias=bias, resid=x)      # C aliases R
    tol = 1e-4 if dtype == torch.float32 else None
    if tol:
        torch.testing.assert_close(x.cpu().double(), ref, atol=tol, rtol=tol)
    else:
        assert rel_err(x, ref) < BF16_REL


def test_gemm_bf16_unaligned_takes_cuda_core_path():
    M, N, K = 40, 70, 36                       # K*2 bytes not a multiple of 16 -> no TMA
    a, w = randn(M, K, seed=18).bfloat16(), randn(N, K, seed=19).bfloat16()
    y = cg.cutile_linear(a.cuda(), w.cuda())
    assert rel_err(y, a.double() @ w.double().t()) < BF16_REL


def test_gemm_rejects_bad_args():
    a = torch.zeros(4, 8, device="cuda")
    w = torch.zeros(4, 8, device="cuda")
    out = torch.zeros(4, 4, device="cuda")
    with pytest.raises(ValueError):
        ops.gemm(a, w, out, epilogue=L.EPI_BIAS)          # bias missing
    with pytest.raises(ValueError):
        ops.gemm(a, w, out, epilogue=9)


# ----------------------------------------------------------------- attention
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,H,T,D", [(2, 3, 32, 16), (2, 4, 128, 64), (1, 12, 100, 64), (2, 6, 256, 64),
                                     (1, 2, 513, 64), (1, 25, 70, 64), (2, 2, 65, 32), (1, 1, 1, 64),
                                     (1, 2, 40, 128)])
def test_attention(dtype, B, H, T, D):
    q, k, v = (randn(B, H, T, D, seed=s).to(dtype) for s in (20, 21, 22))
    y = cg.cutile_causal_attention(q.cuda(), k.cuda(), v.cuda(), H)
    ref = R.causal_attention(q.double(), k.double(), v.double())
    if dtype == torch.float32:
        torch.testing.assert_close(y.cpu().double(), ref, atol=1e-3, rtol=1e-3)
    else:
        assert rel_err(y, ref) < BF16_REL


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_attention_from_fused_qkv_layout(dtype):
    B, T, H, D = 2, 150, 12, 64
    C = H * D
    qkv = randn(B, T, 3 * C, seed=23).to(dtype).cuda()
    q4 = qkv.view(B, T, 3, H, D)
    out = torch.empty((B, T, C), dtype=dtype, device="cuda")
    ops.attention_prefill(q4[:, :, 0].transpose(1, 2), q4[:, :, 1].transpose(1, 2), q4[:, :, 2].transpose(1, 2),
                          out.view(B, T, H, D).transpose(1, 2))
    qc = qkv.cpu().double().view(B, T, 3, H, D)
    ref = R.causal_attention(*(qc[:, :, j].transpose(1, 2) for j in range(3))).transpose(1, 2).reshape(B, T, C)
    if dtype == torch.float32:
        torch.testing.assert_close(out.cpu().double(), ref, atol=1e-3, rtol=1e-3)
    else:
        assert rel_err(out, ref) < BF16_REL


# ----------------------------------------------------------------- KV cache + decode
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,H,D,Tmax,Lq", [(4, 12, 64, 256, 200), (64, 12, 64, 256, 129), (2, 25, 64, 1024, 1000),
                                           (3, 3, 16, 64, 5), (1, 2, 128, 300, 300), (8, 12, 64, 256, 256)])
def test_kv_append_and_decode(dtype, B, H, D, Tmax, Lq):
    C = H * D
    cache_k = torch.zeros((B, H, Tmax, D), dtype=dtype, device="cuda")
    cache_v = torch.zeros_like(cache_k)
    qkv_prompt = randn(B, Lq - 1, 3 * C, seed=30).to(dtype).cuda()
    ops.kv_append(qkv_prompt, cache_k, cache_v, pos0=0)
    qkv_new = randn(B, 3 * C, seed=31).to(dtype).cuda()
    pos = torch.tensor([Lq - 1], dtype=torch.int64, device="cuda")
    ops.kv_append(qkv_new.view(B, 1, 3 * C), cache_k, cache_v, pos0=0, pos_dev=pos)
    allqkv = torch.cat([qkv_prompt.cpu(), qkv_new.cpu().view(B, 1, 3 * C)], 1).double()
    k_ref = allqkv[:, :, C:2 * C].view(B, Lq, H, D).transpose(1, 2)
    v_ref = allqkv[:, :, 2 * C:].view(B, Lq, H, D).transpose(1, 2)
    assert torch.equal(cache_k[:, :, :Lq].cpu().double(), k_ref)
    assert torch.equal(cache_v[:, :, :Lq].cpu().double(), v_ref)
    ws = torch.empty(max(16, ops.decode_workspace_bytes(B, H, D, Tmax)), dtype=torch.uint8, device="cuda")
    out = torch.empty((B, C), dtype=dtype, device="cuda")
    ops.attention_decode(qkv_new[:, :C], cache_k, cache_v, out, 1, ws, len_dev=pos)
    q = qkv_new.cpu().double()[:, :C].view(B, H, 1, D)
    att = torch.softmax((q @ k_ref.transpose(-1, -2)) / math.sqrt(D), dim=-1) @ v_ref
    ref = att.view(B, C)
    if dtype == torch.float32:
        torch.testing.assert_close(out.cpu().double(), ref, atol=1e-4, rtol=1e-4)
    else:
        assert rel_err(out, ref) < BF16_REL
    # host-length form agrees with the device-length form
    out2 = torch.empty_like(out)
    ws2 = torch.empty(max(16, ops.decode_workspace_bytes(B, H, D, Lq)), dtype=torch.uint8, device="cuda")
    ops.attention_decode(qkv_new[:, :C], cache_k, cache_v, out2, Lq, ws2)
    assert rel_err(out2, ref) < (1e-5 if dtype == torch.float32 else BF16_REL)


# ----------------------------------------------------------------- argmax / advance
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_argmax_and_advance(dtype):
    B, V = 5, 50257
    logits = randn(B, V, seed=40).to(dtype)
    logits[2, 17] = logits[2, 40000] = 100.0   # tie -> first index
    big = torch.zeros((B, V + 3), dtype=dtype)
    big[:, :V] = logits
    tok = torch.empty(B, dtype=torch.int64, device="cuda")
    ops.argmax(big.cuda()[:, :V], tok)
    ref = logits.float().argmax(-1)
    assert torch.equal(tok.cpu(), ref)
    assert tok[2].item() == 17
    seq = torch.zeros((B, 10), dtype=torch.int64, device="cuda")
    pos = torch.tensor([3], dtype=torch.int64, device="cuda")
    ops.decode_advance(tok, pos, seq)
    assert pos.item() == 4
    assert torch.equal(seq[:, 4].cpu(), ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_argmax_edge_rows(dtype):
    V = 50257
    x = randn(7, V, seed=41).to(dtype)
    x[0, 5] = x[0, 5 + 1024] = x[0, 5 + 8 * 1024 + 3] = 50.0       # ties across threads / unroll slots
    x[1, :] = float("-inf")                                        # all -inf -> index 0
    x[2, 0] = float("nan"); x[2, 777] = 60.0; x[2, 900] = float("nan")   # NaN never wins
    x[3, V - 1] = 70.0                                             # last element
    x[4, :] = float("nan"); x[4, 12345] = -3.0                     # the only number wins
    x[6, 6282] = x[6, 6283] = x[6, 40000] = 80.0                    # tie across a wide-row chunk boundary
    x[5, 2] = x[5, 10] = 90.0     # row 5 starts 5 elements into a 16-byte unit: tie between its head and a vector
    tok = torch.empty(7, dtype=torch.int64, device="cuda")
    ops.argmax(x.cuda(), tok)
    assert tok.cpu().tolist()[:5] == [5, 0, 777, V - 1, 12345]
    assert tok[5].item() == 2
    assert tok[6].item() == 6282
    small = randn(64, 3, seed=42).to(dtype)
    tok64 = torch.empty(64, dtype=torch.int64, device="cuda")
    ops.argmax(small.cuda(), tok64)
    assert torch.equal(tok64.cpu(), small.float().argmax(-1))


# ----------------------------------------------------------------- few-row (decode) GEMM: cluster split-K
@pytest.mark.parametrize("epi", EPIS)
@pytest.mark.parametrize("M,N,K", [(64, 2304, 768), (64, 768, 3072), (8, 768, 768), (1, 50257, 768),
                                   (200, 3072, 768), (256, 1000, 1600), (17, 130, 48), (64, 768, 768)])
def test_gemm_few_rows(epi, M, N, K):
    dtype = torch.bfloat16
    a = randn(M, K, seed=50).to(dtype).cuda()
    w = (randn(N, K, seed=51) / math.sqrt(K)).to(dtype).cuda()
    bias = randn(N, seed=52).to(dtype).cuda()
    for it in range(2):
        r = randn(M, N, seed=53 + it).to(dtype).cuda()
        ref = gemm_ref(a.cpu(), w.cpu(), bias.cpu(), r.cpu(), epi)
        out = r.clone() if epi == L.EPI_BIAS_RESIDUAL else torch.empty((M, N), dtype=dtype, device="cuda")
        ops.gemm(a, w, out, bias=bias, resid=out if epi == L.EPI_BIAS_RESIDUAL else None, epilogue=epi)
        assert rel_err(out, ref) < BF16_REL, (it, rel_err(out, ref))


# ----------------------------------------------------------------- sampling (temperature / top-k / multinomial)
def _draw(row, n_rows, steps, temperature=1.0, top_k=None, seed=1234):
    """n_rows copies of one logits row, `steps` launches -> all drawn ids (CPU int64)."""
    x = row.view(1, -1).expand(n_rows, -1).contiguous().cuda()
    out = torch.empty(n_rows, dtype=torch.int64, device="cuda")
    seed_t = torch.tensor([seed], dtype=torch.int64, device="cuda")
    got = []
    for s in range(steps):
        ops.sample(x, out, temperature, top_k, seed_t, None, step0=s)
        got.append(out.cpu().clone())
    return torch.cat(got)


def _chi2_ok(counts, probs, n):
    """Pearson chi-square over the support, compared with a loose bound (k - 1 + 6 sqrt(2(k-1)))."""
    exp = probs * n
    k = int((probs > 0).sum())
    stat = (((counts - exp) ** 2) / exp.clamp_min(1e-12))[probs > 0].sum().item()
    return stat < (k - 1) + 6 * math.sqrt(2 * (k - 1)), stat


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("temperature,top_k", [(1.0, None), (0.5, None), (1.0, 3), (2.0, 5)])
def test_sample_distribution(dtype, temperature, top_k):
    V = 50257
    ids = torch.tensor([7, 100, 2048, 30000, 50256, 12, 999, 4444])
    vals = torch.tensor([2.0, 1.5, 1.0, 0.5, 0.0, -0.5, -1.0, -2.0])
    row = torch.full((V,), -40.0)
    row[ids] = vals
    row = row.to(dtype)
    n = 4096 * 6
    got = _draw(row, 4096, 6, temperature, top_k)
    z = row.float()[ids] / temperature
    if top_k is not None:
        z[top_k:] = float("-inf")                       # vals are sorted: the top-k are the first k
    probs = torch.softmax(z.double(), 0)
    assert torch.isin(got, ids[probs > 0]).all()        # mass outside the set (e^-40) never drawn at this n
    counts = torch.stack([(got == i).sum() for i in ids]).double()
    ok, stat = _chi2_ok(counts, probs, n)
    assert ok, (stat, counts, probs * n)


def test_sample_deterministic_in_seed_and_step():
    row = randn(50257, seed=60).bfloat16()
    a = _draw(row, 64, 2, 1.0, 40, seed=5)
    b = _draw(row, 64, 2, 1.0, 40, seed=5)
    c = _draw(row, 64, 2, 1.0, 40, seed=6)
    assert torch.equal(a, b)
    assert not torch.equal(a, c)
    assert not torch.equal(a[:64], a[64:])             # another step draws afresh


def test_sample_edges():
    V = 1000
    x = torch.full((4, V), -5.0)
    x[0, [3, 10, 11]] = torch.tensor([5.0, 3.0, 3.0])  # top_k=2: the tie at the threshold stays in
    x[1, :] = float("-inf")                             # nothing finite -> 0
    x[2, :] = float("nan"); x[2, 77] = 1.0              # NaN never drawn
    x[3, 500] = 50.0                                    # one dominant value
    out = torch.empty(4, dtype=torch.int64, device="cuda")
    seen0 = set()
    seed = torch.tensor([9], dtype=torch.int64, device="cuda")
    for s in range(200):
        ops.sample(x.cuda(), out, 1.0, 2, seed, None, step0=s)
        o = out.cpu().tolist()
        seen0.add(o[0])
        assert o[1] == 0 and o[2] == 77 and o[3] == 500
    assert seen0 == {3, 10, 11}
    with pytest.raises(Exception):
        ops.sample(x.cuda(), out, 0.0, None)


# ----------------------------------------------------------------- fused decode GEMM (LayerNorm fold, row stats, KV)
@pytest.mark.parametrize("M,C,N,epi", [(64, 768, 2304, L.EPI_BIAS), (64, 768, 3072, L.EPI_BIAS_GELU),
                                       (5, 768, 50257, L.EPI_NONE), (130, 1600, 4800, L.EPI_BIAS),
                                       (16, 384, 1536, L.EPI_BIAS_GELU)])
def test_gemm_layernorm_fold(M, C, N, epi):
    """ln_f/ln_1/ln_2 folded into the next GEMM equals LayerNorm then Linear (oracle in fp64)."""
    dt = torch.bfloat16
    x = (randn(M, C, seed=70, scale=2.0) + 0.7).to(dt)           # rows with a nonzero mean
    g = (randn(C, seed=71) * 0.2 + 1.0).to(dt)
    b = (randn(C, seed=72) * 0.2).to(dt)
    w = (randn(N, C, seed=73) / math.sqrt(C)).to(dt)
    bias = randn(N, seed=74).to(dt) if epi != L.EPI_NONE else None
    xc, wc = x.cuda(), w.cuda()
    wf, u, v = ops.lnfold_weights(wc, g.cuda(), b.cuda(), bias.cuda() if bias is not None else None)
    stats = torch.empty((1, M, 2), dtype=torch.float32, device="cuda")
    ops.row_stats(xc, stats)
    out = torch.empty((M, N), dtype=dt, device="cuda")
    ops.gemm_fused(xc, wf, out, epilogue=epi, ln=(stats, 1e-5, u, v))
    h = R.layer_norm(x.double(), g.double(), b.double())
    ref = h @ w.double().t()
    if bias is not None:
        ref = ref + bias.double()
    if epi == L.EPI_BIAS_GELU:
        ref = R.gelu(ref)
    assert rel_err(out, ref) < BF16_REL, rel_err(out, ref)
    s = x.double().sum(-1), (x.double() ** 2).sum(-1)
    torch.testing.assert_close(stats[0].cpu().double(), torch.stack(s, -1), rtol=1e-5, atol=1e-3)


@pytest.mark.parametrize("M,N,K", [(64, 768, 768), (64, 768, 3072), (120, 1600, 6400), (7, 768, 3072)])
def test_gemm_row_stats_of_residual_output(M, N, K):
    dt = torch.bfloat16
    a, w = randn(M, K, seed=75).to(dt).cuda(), (randn(N, K, seed=76) / math.sqrt(K)).to(dt).cuda()
    bias, r = randn(N, seed=77).to(dt).cuda(), randn(M, N, seed=78).to(dt).cuda()
    parts = (N + 127) // 128
    st = torch.full((parts, M, 2), float("nan"), dtype=torch.float32, device="cuda")
    out = torch.empty((M, N), dtype=dt, device="cuda")
    ops.gemm_fused(a, w, out, bias=bias, resid=r, row_stats=st)
    ref = a.double().cpu() @ w.double().cpu().t() + bias.double().cpu() + r.double().cpu()
    assert rel_err(out, ref) < BF16_REL
    o = out.double().cpu()                                          # stats are of the stored bf16 rows
    got = st.double().cpu().sum(0)
    torch.testing.assert_close(got[:, 0], o.sum(-1), rtol=1e-5, atol=1e-2)
    torch.testing.assert_close(got[:, 1], (o ** 2).sum(-1), rtol=1e-5, atol=1e-2)
    for t in range(parts):                                          # each tile covers its own columns
        seg = o[:, t * 128:(t + 1) * 128]
        torch.testing.assert_close(st[t, :, 0].double().cpu(), seg.sum(-1), rtol=1e-5, atol=1e-2)


@pytest.mark.parametrize("B,H", [(64, 12), (3, 25)])
def test_gemm_qkv_kv_append(B, H):
    """The QKV GEMM writes q|k|v and appends k, v to the caches at the device position."""
    dt, D, Tmax = torch.bfloat16, 64, 40
    C = H * D
    x, w = randn(B, C, seed=79).to(dt).cuda(), (randn(3 * C, C, seed=80) / math.sqrt(C)).to(dt).cuda()
    bias = randn(3 * C, seed=81).to(dt).cuda()
    kc = torch.zeros((B, H, Tmax, D), dtype=dt, device="cuda")
    vc = torch.zeros_like(kc)
    pos = torch.tensor([17], dtype=torch.int64, device="cuda")
    qkv = torch.empty((B, 3 * C), dtype=dt, device="cuda")
    ops.gemm_fused(x, w, qkv, bias=bias, kv=(kc, vc, pos, 2))
    ref = x.double().cpu() @ w.double().cpu().t() + bias.double().cpu()
    assert rel_err(qkv, ref) < BF16_REL
    q3 = qkv.view(B, 3, H, D).cpu()
    assert torch.equal(kc[:, :, 19].cpu(), q3[:, 1]) and torch.equal(vc[:, :, 19].cpu(), q3[:, 2])
    kc[:, :, 19] = 0
    vc[:, :, 19] = 0
    assert kc.abs().sum().item() == 0 and vc.abs().sum().item() == 0   # nothing else touched
    with pytest.raises(ValueError):
        ops.gemm_fused(x, w[:100], qkv[:, :100], bias=bias[:100], kv=(kc, vc, pos, 0))   # N != 3 * H * D


# ----------------------------------------------------------------- 16-column decode GEMM (exact fp64 row sums)
@pytest.mark.parametrize("M,C,N,epi", [(64, 768, 2304, L.EPI_BIAS), (64, 768, 3072, L.EPI_BIAS_GELU),
                                       (1, 768, 2304, L.EPI_BIAS), (100, 1600, 4800, L.EPI_BIAS),
                                       (128, 768, 3072, L.EPI_BIAS_GELU), (7, 384, 1536, L.EPI_BIAS_GELU)])
def test_rows_gemm_layernorm_fold_fp64_sums(M, C, N, epi):
    """LayerNorm folded in with exact fp64 row totals (gpt_row_sums) equals LayerNorm then Linear."""
    dt = torch.bfloat16
    x = (randn(M, C, seed=90, scale=2.0) + 0.7).to(dt)
    g = (randn(C, seed=91) * 0.2 + 1.0).to(dt)
    b = (randn(C, seed=92) * 0.2).to(dt)
    w = (randn(N, C, seed=93) / math.sqrt(C)).to(dt)
    bias = randn(N, seed=94).to(dt)
    xc = x.cuda()
    wf, u, v = ops.lnfold_weights(w.cuda(), g.cuda(), b.cuda(), bias.cuda())
    sums = torch.full((M, 2), float("nan"), dtype=torch.float64, device="cuda")
    zero = torch.full((3, M, 2), 5.0, dtype=torch.float64, device="cuda")
    ops.row_sums(xc, sums, zero=zero)
    xd = x.double()
    torch.testing.assert_close(sums.cpu(), torch.stack([xd.sum(-1), (xd ** 2).sum(-1)], -1), rtol=0, atol=1e-9)
    assert zero.abs().sum().item() == 0
    out = torch.empty((M, N), dtype=dt, device="cuda")
    ops.gemm_fused(xc, wf, out, epilogue=epi, ln=(sums, 1e-5, u, v))
    ref = R.layer_norm(xd, g.double(), b.double()) @ w.double().t() + bias.double()
    if epi == L.EPI_BIAS_GELU:
        ref = R.gelu(ref)
    assert rel_err(out, ref) < BF16_REL, rel_err(out, ref)


@pytest.mark.parametrize("M,N,K", [(64, 768, 768), (64, 768, 3072), (100, 1600, 6400), (7, 768, 3072),
                                   (128, 768, 768), (1, 1600, 1600)])
def test_rows_gemm_residual_row_sums_split_k(M, N, K):
    """Residual epilogue in place (C is R) over split-K clusters; fp64 row sums of the stored rows are
    accumulated into what the buffer held (exact, so equal to the fp64 sums of the output + the start)."""
    dt = torch.bfloat16
    a, w = randn(M, K, seed=95).to(dt).cuda(), (randn(N, K, seed=96) / math.sqrt(K)).to(dt).cuda()
    bias, x = randn(N, seed=97).to(dt).cuda(), randn(M, N, seed=98).to(dt).cuda()
    x0 = x.double().cpu()
    sums = torch.zeros((M, 2), dtype=torch.float64, device="cuda")
    sums[:, 0] = 3.0
    ops.gemm_fused(a, w, x, bias=bias, resid=x, row_stats=sums)
    ref = a.double().cpu() @ w.double().cpu().t() + bias.double().cpu() + x0
    assert rel_err(x, ref) < BF16_REL, rel_err(x, ref)
    o = x.double().cpu()
    torch.testing.assert_close(sums[:, 0].cpu(), o.sum(-1) + 3.0, rtol=0, atol=1e-9)
    torch.testing.assert_close(sums[:, 1].cpu(), (o ** 2).sum(-1), rtol=0, atol=1e-9)
    # deterministic: the same call on the same inputs gives bit-identical outputs and sums
    x2 = x0.to(dt).cuda()
    s2 = torch.zeros((M, 2), dtype=torch.float64, device="cuda")
    s2[:, 0] = 3.0
    ops.gemm_fused(a, w, x2, bias=bias, resid=x2, row_stats=s2)
    assert torch.equal(x2, x) and torch.equal(s2, sums)


@pytest.mark.parametrize("B,H", [(64, 12), (3, 25), (128, 12)])
def test_rows_gemm_qkv_kv_append_with_fold(B, H):
    """The folded QKV GEMM writes q|k|v and appends k, v at the device position (16-column kernel)."""
    dt, D, Tmax = torch.bfloat16, 64, 40
    C = H * D
    x = randn(B, C, seed=99).to(dt).cuda()
    g, b = (randn(C, seed=100) * 0.1 + 1).to(dt).cuda(), (randn(C, seed=101) * 0.1).to(dt).cuda()
    w, bias = (randn(3 * C, C, seed=102) / math.sqrt(C)).to(dt).cuda(), randn(3 * C, seed=103).to(dt).cuda()
    wf, u, v = ops.lnfold_weights(w, g, b, bias)
    sums = torch.empty((B, 2), dtype=torch.float64, device="cuda")
    ops.row_sums(x, sums)
    kc = torch.zeros((B, H, Tmax, D), dtype=dt, device="cuda")
    vc = torch.zeros_like(kc)
    pos = torch.tensor([17], dtype=torch.int64, device="cuda")
    qkv = torch.empty((B, 3 * C), dtype=dt, device="cuda")
    ops.gemm_fused(x, wf, qkv, epilogue=L.EPI_BIAS, ln=(sums, 1e-5, u, v), kv=(kc, vc, pos, 2))
    ref = R.layer_norm(x.double().cpu(), g.double().cpu(), b.double().cpu()) @ w.double().cpu().t() \
        + bias.double().cpu()
    assert rel_err(qkv, ref) < BF16_REL
    q3 = qkv.view(B, 3, H, D).cpu()
    assert torch.equal(kc[:, :, 19].cpu(), q3[:, 1]) and torch.equal(vc[:, :, 19].cpu(), q3[:, 2])
    kc[:, :, 19] = 0
    vc[:, :, 19] = 0
    assert kc.abs().sum().item() == 0 and vc.abs().sum().item() == 0


def test_rows_gemm_lm_head_fold_any_n():
    """ln_f folded into a head whose N is not a multiple of 16 (fp64 totals on the few-row kernel)."""
    dt, M, C, N = torch.bfloat16, 64, 768, 50257
    x = randn(M, C, seed=104, scale=1.5).to(dt).cuda()
    g, b = (randn(C, seed=105) * 0.1 + 1).to(dt).cuda(), (randn(C, seed=106) * 0.1).to(dt).cuda()
    w = (randn(N, C, seed=107) / math.sqrt(C)).to(dt).cuda()
    wf, u, v = ops.lnfold_weights(w, g, b, None)
    sums = torch.empty((M, 2), dtype=torch.float64, device="cuda")
    ops.row_sums(x, sums)
    out = torch.empty((M, N), dtype=dt, device="cuda")
    ops.gemm_fused(x, wf, out, epilogue=L.EPI_NONE, ln=(sums, 1e-5, u, v))
    ref = R.layer_norm(x.double().cpu(), g.double().cpu(), b.double().cpu()) @ w.double().cpu().t()
    assert rel_err(out, ref) < BF16_REL
