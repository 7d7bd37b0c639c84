"""Pointer-level wrappers over libgpt_b200 (caller provides every output).

These are what the model's forward / decode loop calls: no allocation, no
copies, the current torch CUDA stream. The reference-named operators in the
sibling modules (``cutile_gelu`` …) allocate their outputs and delegate here.
"""
from __future__ import annotations

import ctypes
import math

import torch

from .. import _lib as L


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _row_stride(t: torch.Tensor, what: str) -> int:
    """Row stride of a 2-D view whose rows are contiguous."""
    if t.dim() != 2 or (t.size(1) > 1 and t.stride(1) != 1):
        raise ValueError(f"{what}: expected a 2-D tensor with contiguous rows, got shape "
                         f"{tuple(t.shape)} strides {t.stride()}")
    return t.stride(0) if t.size(0) > 1 else max(t.size(1), t.stride(0))


def embedding(idx: torch.Tensor, weight: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    n = idx.numel()
    V, C = weight.shape
    L.check(L.lib().gpt_embedding(_ptr(idx), n, _ptr(weight), V, C, _ptr(out),
                                  L.dtype_code(weight.dtype), L.stream_ptr()), "gpt_embedding")
    return out


def embedding_pos(idx: torch.Tensor, wte: torch.Tensor, wpe: torch.Tensor, out: torch.Tensor,
                  pos0: int = 0, pos_dev: torch.Tensor | None = None) -> torch.Tensor:
    """out[b, t] = wte[idx[b, t]] + wpe[pos0 + (*pos_dev) + t] (pos_dev: optional int64 device scalar)."""
    B, T = idx.shape
    V, C = wte.shape
    L.check(L.lib().gpt_embedding_pos(_ptr(idx), B, T, _ptr(wte), _ptr(wpe), V, wpe.shape[0], C, pos0,
                                      _ptr(pos_dev), _ptr(out), L.dtype_code(wte.dtype), L.stream_ptr()),
            "gpt_embedding_pos")
    return out


def layernorm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, out: torch.Tensor,
              eps: float = 1e-5) -> torch.Tensor:
    C = x.shape[-1]
    M = x.numel() // C
    L.check(L.lib().gpt_layernorm(_ptr(x), _ptr(w), _ptr(b), _ptr(out), M, C, float(eps),
                                  L.dtype_code(x.dtype), L.stream_ptr()), "gpt_layernorm")
    return out


def gelu(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    L.check(L.lib().gpt_gelu(_ptr(x), _ptr(out), x.numel(), L.dtype_code(x.dtype), L.stream_ptr()),
            "gpt_gelu")
    return out


def gemm(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor, bias: torch.Tensor | None = None,
         resid: torch.Tensor | None = None, epilogue: int | None = None) -> torch.Tensor:
    """out[M, N] = epilogue(a[M, K] · w[N, K]ᵀ); a/out/resid may be row-strided views."""
    M, K = a.shape
    N = w.shape[0]
    if w.shape[1] != K or not w.is_contiguous():
        raise ValueError(f"gemm: weight must be a contiguous [N, K={K}] tensor, got {tuple(w.shape)}")
    if epilogue is None:
        epilogue = (L.EPI_NONE if bias is None else
                    L.EPI_BIAS if resid is None else L.EPI_BIAS_RESIDUAL)
    lda = _row_stride(a, "gemm A")
    ldc = _row_stride(out, "gemm C")
    ldr = _row_stride(resid, "gemm residual") if resid is not None else 0
    L.check(L.lib().gpt_gemm(_ptr(a), lda, _ptr(w), _ptr(bias), _ptr(resid), ldr, _ptr(out), ldc, M, N, K,
                             epilogue, L.dtype_code(a.dtype), L.stream_ptr()), "gpt_gemm")
    return out


def gemm_fused(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor, bias: torch.Tensor | None = None,
               resid: torch.Tensor | None = None, epilogue: int | None = None, ln=None,
               row_stats: torch.Tensor | None = None, kv=None) -> torch.Tensor:
    """Few-row (decode) GEMM with fused extras, bf16, M <= 256.

    ln = (stats, eps, u [N] fp32, v [N] fp32): LayerNorm folded in, `w` being the gamma-scaled
    weight from lnfold_weights; stats is either fp64 [M, 2] exact row totals or fp32 [parts, M, 2]
    per-tile sums. row_stats fp64 [M, 2] is added to with the (sum, sum of squares) of the stored
    rows (the 16-column decode GEMM); fp32 [ceil(N/128), M, 2] receives per-tile sums instead.
    kv = (k_cache, v_cache [B, H, Tmax, D], pos_dev int64 [1] or None, pos0) appends the k / v
    parts of a fused QKV output.
    """
    M, K = a.shape
    N = w.shape[0]
    if w.shape[1] != K or not w.is_contiguous():
        raise ValueError(f"gemm_fused: weight must be a contiguous [N, K={K}] tensor, got {tuple(w.shape)}")
    if epilogue is None:
        epilogue = (L.EPI_NONE if bias is None and ln is None else
                    L.EPI_BIAS if resid is None else L.EPI_BIAS_RESIDUAL)
    f = L.GemmFusion()
    if ln is not None:
        stats, eps, u, v = ln
        f.ln_eps, f.ln_u, f.ln_v = float(eps), _ptr(u), _ptr(v)
        if stats.dtype == torch.float64:         # exact row totals [M, 2]
            f.ln_sums = _ptr(stats)
        else:                                    # fp32 per-tile parts [parts, M, 2]
            f.ln_stats, f.ln_parts = _ptr(stats), stats.shape[0]
    if row_stats is not None:
        if row_stats.dtype == torch.float64:     # [M, 2], accumulated into
            f.row_sums = _ptr(row_stats)
        else:
            f.row_stats = _ptr(row_stats)
    if kv is not None:
        kc, vc, pos_dev, pos0 = kv
        _, H, Tmax, D = kc.shape
        f.k_cache, f.v_cache, f.kv_heads, f.kv_dim, f.kv_tmax = _ptr(kc), _ptr(vc), H, D, Tmax
        f.kv_pos0, f.kv_pos_dev = int(pos0), _ptr(pos_dev)
    lda = _row_stride(a, "gemm A")
    ldc = _row_stride(out, "gemm C")
    ldr = _row_stride(resid, "gemm residual") if resid is not None else 0
    L.check(L.lib().gpt_gemm_fused(_ptr(a), lda, _ptr(w), _ptr(bias), _ptr(resid), ldr, _ptr(out), ldc, M, N, K,
                                   epilogue, ctypes.byref(f), L.dtype_code(a.dtype), L.stream_ptr()),
            "gpt_gemm_fused")
    return out


def row_stats(x: torch.Tensor, stats: torch.Tensor) -> torch.Tensor:
    """stats [1, M, 2] fp32 <- (sum, sum of squares) of each row of x [M, C]."""
    M, C = x.shape
    L.check(L.lib().gpt_row_stats(_ptr(x), _row_stride(x, "row_stats"), M, C, _ptr(stats), L.dtype_code(x.dtype),
                                  L.stream_ptr()), "gpt_row_stats")
    return stats


def row_sums(x: torch.Tensor, sums: torch.Tensor, zero: torch.Tensor | None = None) -> torch.Tensor:
    """sums fp64 [M, 2] <- (sum, sum of squares) of each row of x [M, C]; `zero` (fp64, any shape,
    contiguous) is cleared in the same launch."""
    M, C = x.shape
    nz = zero.numel() if zero is not None else 0
    L.check(L.lib().gpt_row_sums(_ptr(x), _row_stride(x, "row_sums"), M, C, _ptr(sums), _ptr(zero), nz,
                                 L.dtype_code(x.dtype), L.stream_ptr()), "gpt_row_sums")
    return sums


def lnfold_weights(w: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, bias: torch.Tensor | None):
    """LayerNorm fold of Linear w [N, K]: (w * gamma, u [N] fp32, v [N] fp32), see gpt_lnfold_weights."""
    N, K = w.shape
    wf = torch.empty_like(w)
    u = torch.empty(N, dtype=torch.float32, device=w.device)
    v = torch.empty(N, dtype=torch.float32, device=w.device)
    L.check(L.lib().gpt_lnfold_weights(_ptr(w), _ptr(gamma), _ptr(beta), _ptr(bias), N, K, _ptr(wf), _ptr(u),
                                       _ptr(v), L.dtype_code(w.dtype), L.stream_ptr()), "gpt_lnfold_weights")
    return wf, u, v


def attention_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                      scale: float | None = None) -> torch.Tensor:
    """Causal attention over 4-D views indexed [B, H, T, D] (any b/h/t strides, d contiguous)."""
    B, H, T, D = q.shape
    for t, name in ((q, "q"), (k, "k"), (v, "v"), (out, "out")):
        if t.shape != (B, H, T, D) or (D > 1 and t.stride(3) != 1):
            raise ValueError(f"attention: {name} must be a [B,H,T,D] view with contiguous D")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    st = [L.strides3(*t.stride()[:3]) for t in (q, k, v, out)]
    L.check(L.lib().gpt_attention_prefill(_ptr(q), _ptr(k), _ptr(v), _ptr(out), B, H, T, D, st[0], st[1],
                                          st[2], st[3], float(scale), L.dtype_code(q.dtype),
                                          L.stream_ptr()), "gpt_attention_prefill")
    return out


def kv_append(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, pos0: int = 0,
              pos_dev: torch.Tensor | None = None) -> None:
    """qkv [B, Tn, 3C] (row stride may exceed 3C) -> caches [B, H, Tmax, D] at pos0 (+ *pos_dev)."""
    B, Tn, C3 = qkv.shape
    _, H, Tmax, D = k_cache.shape
    ld = qkv.stride(1) if Tn > 1 else qkv.stride(0) if B > 1 else C3
    L.check(L.lib().gpt_kv_append(_ptr(qkv), ld, _ptr(k_cache), _ptr(v_cache), B, H, Tn, D, Tmax, pos0,
                                  _ptr(pos_dev), L.dtype_code(qkv.dtype), L.stream_ptr()), "gpt_kv_append")


def decode_workspace_bytes(B: int, H: int, D: int, Lmax: int) -> int:
    return int(L.lib().gpt_attention_decode_workspace_size(B, H, D, Lmax))


def attention_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, out: torch.Tensor,
                     length: int, workspace: torch.Tensor | None, scale: float | None = None,
                     len_dev: torch.Tensor | None = None) -> torch.Tensor:
    """q: [B, >=H*D] rows (e.g. the q third of a [B, 3C] QKV row); out: [B, H*D] rows.

    Attends to the first ``length + (*len_dev)`` cached positions.
    """
    B, H, Tmax, D = k_cache.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    L.check(L.lib().gpt_attention_decode(_ptr(q), _row_stride(q, "decode q"), _ptr(k_cache), _ptr(v_cache),
                                         _ptr(out), _row_stride(out, "decode out"), B, H, D, Tmax, length,
                                         _ptr(len_dev), float(scale), _ptr(workspace), L.dtype_code(q.dtype),
                                         L.stream_ptr()), "gpt_attention_decode")
    return out


def argmax(logits: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """logits [B, V] (row-strided view ok) -> out int64 [B]."""
    B, V = logits.shape
    L.check(L.lib().gpt_argmax(_ptr(logits), _row_stride(logits, "argmax"), B, V, _ptr(out),
                               L.dtype_code(logits.dtype), L.stream_ptr()), "gpt_argmax")
    return out


def sample(logits: torch.Tensor, out: torch.Tensor, temperature: float = 1.0, top_k: int | None = None,
           seed_dev: torch.Tensor | None = None, step_dev: torch.Tensor | None = None, step0: int = 0) -> torch.Tensor:
    """logits [B, V] -> out int64 [B]: temperature, top-k and a multinomial draw in one kernel.

    The draw of row b is fixed by (seed_dev[0], b, step0 + step_dev[0]); both tensors are int64 on the
    device (or None = 0), so the call can be captured in a CUDA graph.
    """
    B, V = logits.shape
    k = 0 if top_k is None else int(top_k)
    L.check(L.lib().gpt_sample(_ptr(logits), _row_stride(logits, "sample"), B, V, float(temperature), k,
                               _ptr(seed_dev), _ptr(step_dev), int(step0), _ptr(out),
                               L.dtype_code(logits.dtype), L.stream_ptr()), "gpt_sample")
    return out


def decode_advance(tok: torch.Tensor, pos_dev: torch.Tensor, seq: torch.Tensor | None = None) -> None:
    """seq[b, *pos_dev + 1] = tok[b]; *pos_dev += 1 (one tiny kernel)."""
    B = tok.numel()
    ld, n = (seq.stride(0), seq.shape[1]) if seq is not None else (0, 0)
    L.check(L.lib().gpt_decode_advance(_ptr(tok), B, _ptr(seq), ld, n, _ptr(pos_dev), L.stream_ptr()),
            "gpt_decode_advance")
