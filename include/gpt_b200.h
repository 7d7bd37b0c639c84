/*
 * gpt_b200.h — C ABI of libgpt_b200.so, the sm_100a (B200) kernel library
 * behind cutilegpt_b200's drop-in replacement of cutileGPT's kernel package.
 *
 * Conventions (every entry point):
 *   - Pointers are CUDA device pointers unless stated otherwise; shapes and
 *     strides are int64 element counts; `stream` is a cudaStream_t passed as
 *     void* (NULL = legacy default stream).
 *   - The library never allocates outputs and never synchronises the stream.
 *     Kernels are launched asynchronously on `stream`.
 *   - Return value is a gpt_status. On failure gpt_last_error_string()
 *     (thread-local) describes the cause. No C++ exception crosses the ABI.
 *   - dtype is a gpt_dtype value; inputs and outputs of one call share it.
 *
 * The Python operator each entry point replaces is cited as
 * `file:line` inside the reference project cutileGPT (package cutile_gpt).
 */
#ifndef GPT_B200_H
#define GPT_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define GPT_API __attribute__((visibility("default")))
#else
#define GPT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  GPT_OK = 0,
  GPT_ERR_SHAPE = 1,        /* inconsistent or out-of-range sizes          */
  GPT_ERR_ALIGN = 2,        /* pointer/stride alignment the kernel needs   */
  GPT_ERR_DTYPE = 3,        /* dtype not supported by this entry point     */
  GPT_ERR_UNSUPPORTED = 4,  /* valid request this build cannot serve       */
  GPT_ERR_CUDA = 5,         /* a CUDA runtime/driver call failed           */
  GPT_ERR_TIMEOUT = 6,      /* a bounded device wait gave up               */
  GPT_ERR_ARG = 7           /* null pointer or bad enum                    */
} gpt_status;

typedef enum { GPT_F32 = 0, GPT_BF16 = 1 } gpt_dtype;

typedef enum {
  GPT_EPI_NONE = 0,           /* C = A·Wᵀ                                  */
  GPT_EPI_BIAS = 1,           /* C = A·Wᵀ + bias                           */
  GPT_EPI_BIAS_GELU = 2,      /* C = gelu_tanh(A·Wᵀ + bias)                */
  GPT_EPI_BIAS_RESIDUAL = 3   /* C = A·Wᵀ + bias + R   (C may alias R)     */
} gpt_epilogue;

/* ---- library / error state ------------------------------------------- */
GPT_API int gpt_version(void);
GPT_API const char* gpt_last_error_string(void);
/* Reads and clears the device-side error word that bounded waits set when
 * they give up (GPT_ERR_TIMEOUT). Synchronises the current device. */
GPT_API int gpt_device_error(int* code_out);
/* Limit, in ns, of every bounded device wait of the library's kernels on
 * the current device (default 4 s). No reference counterpart: the
 * reference's kernels have no bounded waits. Tests shorten it to make a
 * wait run out; it is a library setting, not a GPU setting. */
GPT_API int gpt_set_wait_limit_ns(uint64_t ns);
/* Self-test of the bounded wait (no reference counterpart): one CTA waits
 * on an mbarrier that expects `expected` arrivals (1..32) after making
 * `arrivals` of them. With arrivals < expected the wait runs out after the
 * current limit, the kernel returns, *out_dev = 0 and the next
 * gpt_device_error() reports GPT_ERR_TIMEOUT; otherwise *out_dev = 1.
 * out_dev is one device int. */
GPT_API int gpt_selftest_wait(int expected, int arrivals, int* out_dev, void* stream);
/* Number of SMs of the current device (0 if no device). */
GPT_API int gpt_sm_count(void);
/* Kernels this thread has launched through the library so far. */
GPT_API int64_t gpt_launch_count(void);

/* ---- embedding --------------------------------------------------------- */
/* out[i, :] = weight[idx[i], :] for i < n_idx.  Indices outside [0, vocab)
 * produce GPT_ERR_SHAPE at the next gpt_device_error() and zero rows.
 * Replaces cutile_embedding  (cutile_gpt/kernels/embedding.py:54-109). */
GPT_API int gpt_embedding(const int64_t* idx, int64_t n_idx, const void* weight,
                  int64_t vocab, int64_t C, void* out, int dtype, void* stream);

/* out[b, t, :] = wte[idx[b, t], :] + wpe[p0 + t, :] — the token +
 * position embedding and broadcast add of CutileGPT.forward
 * (cutile_gpt/models/gpt.py:110-113) in one pass. idx is [B, T] contiguous.
 * p0 = pos0 + (pos_dev ? *pos_dev : 0): pos_dev is an optional device-side
 * position so a captured decode step can advance without new arguments.
 * Out-of-range token ids or positions give zero rows and are reported by
 * gpt_device_error(). */
GPT_API int gpt_embedding_pos(const int64_t* idx, int64_t B, int64_t T,
                      const void* wte, const void* wpe, int64_t vocab,
                      int64_t n_pos, int64_t C, int64_t pos0,
                      const int64_t* pos_dev, void* out, int dtype,
                      void* stream);

/* ---- layernorm --------------------------------------------------------- */
/* y[m, :] = (x[m, :] - mean) * rsqrt(var + eps) * w + b over rows of length
 * C (contiguous rows). Statistics in fp32. y may alias x.
 * Replaces cutile_layer_norm (cutile_gpt/kernels/layernorm.py:77-135). */
GPT_API int gpt_layernorm(const void* x, const void* w, const void* b, void* y,
                  int64_t M, int64_t C, float eps, int dtype, void* stream);

/* ---- gelu -------------------------------------------------------------- */
/* y = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), n elements, y may
 * alias x. Replaces cutile_gelu (cutile_gpt/kernels/gelu.py:71-110). */
GPT_API int gpt_gelu(const void* x, void* y, int64_t n, int dtype, void* stream);

/* ---- dense contraction -------------------------------------------------- */
/* C[m, n] = epilogue(sum_k A[m, k] * W[n, k]) with A [M, K] (row stride lda),
 * W [N, K] (the nn.Linear [out, in] layout, contiguous), C [M, N] (row
 * stride ldc), R [M, N] (row stride ldr).  bf16: tcgen05/TMEM tensor-core
 * kernel fed by TMA, fp32 accumulation; f32: fp32 CUDA-core kernel.
 * Replaces cutile_linear / cutile_linear_bias
 * (cutile_gpt/kernels/linear.py:112-161, :164-222) and the residual adds
 * of CutileGPT.forward (cutile_gpt/models/gpt.py:155, :174). */
GPT_API int gpt_gemm(const void* A, int64_t lda, const void* W, const void* bias,
             const void* R, int64_t ldr, void* C, int64_t ldc, int64_t M,
             int64_t N, int64_t K, int epilogue, int dtype, void* stream);

/* ---- attention ----------------------------------------------------------- */
/* Causal softmax(q kᵀ * scale) v for every (b, h).  Element (b, h, t, d) of
 * tensor X lives at X + b*sb + h*sh + t*st + d (d contiguous); q, k, v and
 * out each carry their own strides so both the [B, H, T, D] layout of the
 * reference API and the fused [B, T, 3C] QKV-buffer layout are served
 * without copies. Replaces cutile_causal_attention
 * (cutile_gpt/kernels/attention.py:119-175). */
GPT_API int gpt_attention_prefill(const void* q, const void* k, const void* v,
                          void* out, int64_t B, int64_t H, int64_t T,
                          int64_t D, const int64_t* q_strides,
                          const int64_t* k_strides, const int64_t* v_strides,
                          const int64_t* o_strides, float scale, int dtype,
                          void* stream);

/* ---- KV cache + decode (no reference counterpart: the reference re-runs
 * the full forward per generated token, cutile_gpt/models/gpt.py:204-206) */
/* Copies K and V of Tn new positions from a [B, Tn, 3C] QKV buffer (row
 * stride ld_qkv) into k_cache/v_cache [B, H, Tmax, D] at positions
 * p0..p0+Tn-1, p0 = pos0 + (pos_dev ? *pos_dev : 0). Positions past Tmax
 * are dropped and reported by gpt_device_error(). */
GPT_API int gpt_kv_append(const void* qkv, int64_t ld_qkv, void* k_cache,
                  void* v_cache, int64_t B, int64_t H, int64_t Tn,
                  int64_t D, int64_t Tmax, int64_t pos0,
                  const int64_t* pos_dev, int dtype, void* stream);

/* Bytes of workspace gpt_attention_decode needs when the attended length
 * is at most L (size it with L = Tmax to cover every decode step). */
GPT_API int64_t gpt_attention_decode_workspace_size(int64_t B, int64_t H, int64_t D,
                                            int64_t L);

/* One-query attention per (b, h) over the first Leff cached positions,
 * Leff = L + (len_dev ? *len_dev : 0):
 * out[b, h*D + d] = softmax(q·Kᵀ * scale) V.  q is read from
 * q + b*ld_q + h*D, the caches are [B, H, Tmax, D], out is [B, H*D] with
 * row stride ld_out. Split over the KV length (flash-decoding); partials go
 * to `workspace` (gpt_attention_decode_workspace_size(B, H, D, Lsplit)
 * bytes, Lsplit = L without len_dev and Tmax with it; may be NULL when
 * that size is 0). */
GPT_API int gpt_attention_decode(const void* q, int64_t ld_q, const void* k_cache,
                         const void* v_cache, void* out, int64_t ld_out,
                         int64_t B, int64_t H, int64_t D, int64_t Tmax,
                         int64_t L, const int64_t* len_dev, float scale,
                         void* workspace, int dtype, void* stream);

/* Same computation as gpt_attention_decode, for callers that cannot
 * allocate device memory (fixed-arena runtimes, plugins barred from calling
 * cudaMalloc after start-up, latency-critical loops that must not enter the
 * driver's allocator). No counterpart in the reference, which has no decode
 * path. Instead of a caller workspace, the split-KV partials go to a fixed
 * GPT_NOALLOC_DECODE_SCRATCH_BYTES array inside the library (one per GPU,
 * held from library load until exit); sizes whose
 * gpt_attention_decode_workspace_size exceeds it return GPT_ERR_SHAPE. The
 * first call on a device looks up that array's device address, so make it
 * before any stream capture on that device; the address stays cached until
 * the process exits, so do not call this entry point on a device after
 * cudaDeviceReset(). All calls on a device share the
 * array: calls whose kernels may overlap on the GPU race on it. Nothing in
 * it needs clearing between calls. Allocates nothing. */
#define GPT_NOALLOC_DECODE_SCRATCH_BYTES (256 * 1024)
GPT_API int gpt_attention_decode_noalloc(const void* q, int64_t ld_q,
                         const void* k_cache, const void* v_cache, void* out,
                         int64_t ld_out, int64_t B, int64_t H, int64_t D,
                         int64_t Tmax, int64_t L, const int64_t* len_dev,
                         float scale, int dtype, void* stream);

/* End of a decode step: seq[b, *pos_dev + 1] = tok[b] for b < B (seq row
 * stride ld_seq, skipped when seq is NULL), then *pos_dev += 1. Positions
 * at or past seq_len are not written. One tiny kernel. */
GPT_API int gpt_decode_advance(const int64_t* tok, int64_t B, int64_t* seq,
                       int64_t ld_seq, int64_t seq_len, int64_t* pos_dev,
                       void* stream);

/* out[b] = argmax_v logits[b, v] (first index on ties), logits row stride
 * ld. Greedy step of generate(top_k=1) (cutile_gpt/models/gpt.py:207-225). */
GPT_API int gpt_argmax(const void* logits, int64_t ld, int64_t B, int64_t V,
               int64_t* out, int dtype, void* stream);

/* ---- fused decode GEMM (few rows: M <= 256, bf16) ---------------------
 * Optional extras of gpt_gemm for the KV-cache decode step; every pointer may
 * be NULL (extra off).
 *  - LayerNorm folded into the GEMM (replaces ln_1 / ln_2 / ln_f + GEMM of
 *    cutile_gpt/models/gpt.py:121-130, :158-167, :177-181): A holds the raw
 *    rows x, W the gamma-scaled weight W' = W * gamma (gpt_lnfold_weights),
 *    C = rstd * (x W'^T - mean * ln_u) + ln_v (+ GELU), with mean / rstd of
 *    each row of x from ln_stats [ln_parts][M][2] (sum, sum of squares),
 *    var = E[x^2] - mean^2 as cutile_gpt/kernels/layernorm.py:58-62, and
 *    ln_eps. The bias argument is unused (ln_v holds W . beta + bias).
 *  - row_stats: per 128-column tile, the (sum, sum of squares) of every
 *    stored output row -> row_stats [ceil(N / 128)][M][2]: the ln_stats of
 *    the next folded GEMM (residual stream after attn c_proj / mlp c_proj).
 *  - k_cache / v_cache: the output is the fused QKV row [q | k | v] of
 *    kv_heads x kv_dim each; its k and v parts are also written to the caches
 *    [M][kv_heads][kv_tmax][kv_dim] at position kv_pos0 + *kv_pos_dev
 *    (replaces gpt_kv_append).
 *  - ln_sums / row_sums: the same two extras with exact fp64 row totals
 *    instead of fp32 per-tile parts: ln_sums [M][2] (sum, sum of squares of
 *    each row of x over K) feeds the LayerNorm fold (ln_stats must then be
 *    NULL); row_sums [M][2] is ADDED to (atomically, in fp64, order-free
 *    because the terms are exact) with the (sum, sum of squares) of every
 *    stored output row, so it must hold zeros first (gpt_row_sums clears a
 *    step's worth). With M <= 128, N % 16 == 0 and 16 | kv_dim these run on
 *    the decode-step GEMM with 16-column tiles (gemm_rows); ln_sums alone
 *    also works with any N on M <= 256 (the lm_head). */
typedef struct gpt_gemm_fusion {
  const float* ln_stats;
  int64_t ln_parts;
  float ln_eps;
  const float* ln_u;
  const float* ln_v;
  float* row_stats;
  void* k_cache;
  void* v_cache;
  int64_t kv_heads;
  int64_t kv_dim;
  int64_t kv_tmax;
  int64_t kv_pos0;
  const int64_t* kv_pos_dev;
  const double* ln_sums;
  double* row_sums;
} gpt_gemm_fusion;

GPT_API int gpt_gemm_fused(const void* A, int64_t lda, const void* W,
               const void* bias, const void* R, int64_t ldr, void* C,
               int64_t ldc, int64_t M, int64_t N, int64_t K, int epilogue,
               const gpt_gemm_fusion* fusion, int dtype, void* stream);

/* Start of a folded decode step: sums[m] = (sum, sum of squares) over the
 * C values of row m of x (row stride ld), in fp64 — the ln_sums of the
 * first folded GEMM — and zero[0 .. n_zero) cleared (the row_sums
 * accumulators of the step's later GEMMs). One launch. */
GPT_API int gpt_row_sums(const void* x, int64_t ld, int64_t M, int64_t C,
               double* sums, double* zero, int64_t n_zero, int dtype,
               void* stream);

/* (sum, sum of squares) of each row of x [M, C] (row stride ld) ->
 * stats [1][M][2]: the ln_stats of a folded GEMM that reads the embedding
 * output directly. */
GPT_API int gpt_row_stats(const void* x, int64_t ld, int64_t M, int64_t C,
               float* stats, int dtype, void* stream);

/* LayerNorm fold of a Linear [N, K] that follows LayerNorm(gamma, beta):
 * Wf = W * gamma (per input column, rounded to dtype), u[n] = sum_k Wf[n,k],
 * v[n] = sum_k W[n,k] * beta[k] + bias[n] (bias may be NULL), u / v fp32. */
GPT_API int gpt_lnfold_weights(const void* W, const void* gamma,
               const void* beta, const void* bias, int64_t N, int64_t K,
               void* Wf, float* u, float* v, int dtype, void* stream);

/* Sampling step of generate() with temperature / top_k
 * (cutile_gpt/models/gpt.py:207-225: logits / temperature, top-k mask of
 * values below the k-th largest, softmax, multinomial draw), one launch for
 * all B rows: out[b] = drawn token id. top_k <= 0 or >= V keeps every value;
 * temperature must be > 0. The uniform of row b is a function of
 * (*seed_dev, b, step0 + *step_dev) (SplitMix64), so equal inputs draw equal
 * tokens and a captured CUDA graph draws fresh ones as *step_dev advances;
 * seed_dev / step_dev may be NULL (read as 0). Parity with the reference is
 * distributional (its CuPy RNG stream cannot be reproduced). */
GPT_API int gpt_sample(const void* logits, int64_t ld, int64_t B, int64_t V,
               float temperature, int64_t top_k, const uint64_t* seed_dev,
               const int64_t* step_dev, int64_t step0, int64_t* out, int dtype,
               void* stream);

#ifdef __cplusplus
}
#endif
#endif /* GPT_B200_H */
