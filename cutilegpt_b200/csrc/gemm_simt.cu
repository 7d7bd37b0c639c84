// fp32 CUDA-core contraction C = epilogue(A · Wᵀ) for the fp32 model
// configurations (BASELINE nano / small fp32), where logits must stay within
// max-abs 1e-3 of the reference. The reference multiplies fp32 inputs in
// TF32 (cutile_gpt/kernels/linear.py:61); plain fp32 FFMA is used here so
// the tolerance holds with margin. Also serves bf16 requests the TMA path
// cannot take (unaligned rows), with fp32 accumulation.
//
// Tile 128x128x8, 256 threads, 8x8 outputs per thread, register-prefetched
// double buffering of the shared-memory tiles.
#include "common.cuh"

namespace gpt {
namespace simt {

constexpr int BM = 128, BN = 128, BK = 8, kThreads = 256;

template <typename T, int EPI>
__global__ void __launch_bounds__(kThreads) gemm_simt_kernel(const T* __restrict__ A, int64_t lda,
                                                             const T* __restrict__ W,
                                                             const T* __restrict__ bias,
                                                             const T* R, int64_t ldr, T* C,
                                                             int64_t ldc, int M, int N, int K) {
  pdl_wait();
  pdl_trigger();
  __shared__ float As[2][BK][BM + 4];
  __shared__ float Ws[2][BK][BN + 4];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  // Loader mapping: each thread loads 4 rows x 1 k of A and of W.
  const int lk = tid & 7;         // k within tile
  const int lr = tid >> 3;        // 0..31, rows lr + 32*i
  float ra[4], rw[4];
  auto gload = [&](int k0) {
    int k = k0 + lk;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int m = m0 + lr + 32 * i, n = n0 + lr + 32 * i;
      ra[i] = (m < M && k < K) ? Tr<T>::to_f(A[(int64_t)m * lda + k]) : 0.f;
      rw[i] = (n < N && k < K) ? Tr<T>::to_f(W[(int64_t)n * K + k]) : 0.f;
    }
  };
  auto sstore = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      As[buf][lk][lr + 32 * i] = ra[i];
      Ws[buf][lk][lr + 32 * i] = rw[i];
    }
  };
  const int ty = tid >> 4, tx = tid & 15;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int nk = (K + BK - 1) / BK;
  gload(0);
  sstore(0);
  __syncthreads();
  for (int kt = 0; kt < nk; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < nk) gload((kt + 1) * BK);
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[buf][k][ty * 4 + i];
        a[i + 4] = As[buf][k][64 + ty * 4 + i];
        b[i] = Ws[buf][k][tx * 4 + i];
        b[i + 4] = Ws[buf][k][64 + tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (kt + 1 < nk) sstore(buf ^ 1);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (n >= N) continue;
      float v = acc[i][j];
      if (EPI != GPT_EPI_NONE) v += Tr<T>::to_f(bias[n]);
      if (EPI == GPT_EPI_BIAS_GELU) v = gelu_tanh<false>(v);
      if (EPI == GPT_EPI_BIAS_RESIDUAL) v += Tr<T>::to_f(R[(int64_t)m * ldr + n]);
      C[(int64_t)m * ldc + n] = Tr<T>::from_f(v);
    }
  }
}

template <typename T>
int gemm(const void* A, int64_t lda, const void* W, const void* bias, const void* R, int64_t ldr,
         void* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int epi, cudaStream_t st) {
  if ((M + BM - 1) / BM > 65535) return fail(GPT_ERR_UNSUPPORTED, "gemm_simt: M too large");
  dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM));
  const T *a = (const T*)A, *w = (const T*)W, *b = (const T*)bias, *r = (const T*)R;
  T* c = (T*)C;
  switch (epi) {
    case GPT_EPI_NONE:
      launch_pdl(gemm_simt_kernel<T, GPT_EPI_NONE>, dim3(grid), dim3(kThreads), 0, st, a, lda, w, b, r, ldr, c, ldc, (int)M, (int)N, (int)K);
      break;
    case GPT_EPI_BIAS:
      launch_pdl(gemm_simt_kernel<T, GPT_EPI_BIAS>, dim3(grid), dim3(kThreads), 0, st, a, lda, w, b, r, ldr, c, ldc, (int)M, (int)N, (int)K);
      break;
    case GPT_EPI_BIAS_GELU:
      launch_pdl(gemm_simt_kernel<T, GPT_EPI_BIAS_GELU>, dim3(grid), dim3(kThreads), 0, st, a, lda, w, b, r, ldr, c, ldc, (int)M, (int)N, (int)K);
      break;
    default:
      launch_pdl(gemm_simt_kernel<T, GPT_EPI_BIAS_RESIDUAL>, dim3(grid), dim3(kThreads), 0, st, a, lda, w, b, r, ldr, c, ldc, (int)M, (int)N, (int)K);
      break;
  }
  return launch_status("gemm_simt");
}

}  // namespace simt
}  // namespace gpt

extern "C" int gpt_gemm(const void* A, int64_t lda, const void* W, const void* bias, const void* R,
                        int64_t ldr, void* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int epilogue,
                        int dtype, void* stream) {
  GPT_CHECK_DTYPE(dtype);
  GPT_CHECK_ARG(epilogue >= GPT_EPI_NONE && epilogue <= GPT_EPI_BIAS_RESIDUAL, "gpt_gemm: bad epilogue %d",
                epilogue);
  GPT_CHECK_SHAPE(M >= 0 && N >= 0 && K >= 0 && M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31),
                  "gpt_gemm: bad sizes M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  GPT_CHECK_SHAPE(lda >= K && ldc >= N && (epilogue != GPT_EPI_BIAS_RESIDUAL || ldr >= N),
                  "gpt_gemm: leading dimension smaller than the row");
  if (M == 0 || N == 0) return GPT_OK;
  GPT_CHECK_ARG(A && W && C, "gpt_gemm: null operand");
  GPT_CHECK_ARG(epilogue == GPT_EPI_NONE || bias, "gpt_gemm: epilogue needs bias");
  GPT_CHECK_ARG(epilogue != GPT_EPI_BIAS_RESIDUAL || R, "gpt_gemm: residual epilogue needs R");
  GPT_CHECK_SHAPE(K > 0, "gpt_gemm: K must be positive");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == GPT_BF16) {
    if (gpt::tc::tc_eligible(A, lda, W, K, M, N)) {
      if (M <= gpt::tc::kSkMaxM)
        return gpt::tc::gemm_skinny(A, lda, W, bias, R, ldr, C, ldc, M, N, K, epilogue, st);
      return gpt::tc::gemm_bf16(A, lda, W, bias, R, ldr, C, ldc, M, N, K, epilogue, st, nullptr);
    }
    return gpt::simt::gemm<__nv_bfloat16>(A, lda, W, bias, R, ldr, C, ldc, M, N, K, epilogue, st);
  }
  return gpt::simt::gemm<float>(A, lda, W, bias, R, ldr, C, ldc, M, N, K, epilogue, st);
}

extern "C" int gpt_gemm_fused(const void* A, int64_t lda, const void* W, const void* bias, const void* R,
                              int64_t ldr, void* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int epilogue,
                              const gpt_gemm_fusion* fusion, int dtype, void* stream) {
  if (!fusion) return gpt_gemm(A, lda, W, bias, R, ldr, C, ldc, M, N, K, epilogue, dtype, stream);
  const gpt_gemm_fusion& f = *fusion;
  GPT_CHECK_ARG(dtype == GPT_BF16, "gpt_gemm_fused: bf16 only");
  GPT_CHECK_ARG(epilogue >= GPT_EPI_NONE && epilogue <= GPT_EPI_BIAS_RESIDUAL, "gpt_gemm_fused: bad epilogue %d",
                epilogue);
  GPT_CHECK_SHAPE(M >= 0 && N >= 0 && K > 0 && M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31),
                  "gpt_gemm_fused: bad sizes (M=%lld N=%lld K=%lld)", (long long)M, (long long)N, (long long)K);
  GPT_CHECK_SHAPE(lda >= K && ldc >= N && (epilogue != GPT_EPI_BIAS_RESIDUAL || ldr >= N),
                  "gpt_gemm_fused: leading dimension smaller than the row");
  if (M == 0 || N == 0) return GPT_OK;
  GPT_CHECK_ARG(A && W && C, "gpt_gemm_fused: null operand");
  GPT_CHECK_ARG(epilogue != GPT_EPI_BIAS_RESIDUAL || R, "gpt_gemm_fused: residual epilogue needs R");
  if (f.ln_stats) {
    GPT_CHECK_ARG(f.ln_u && f.ln_v && f.ln_parts >= 1 && f.ln_eps >= 0.f, "gpt_gemm_fused: incomplete LayerNorm fold");
    GPT_CHECK_ARG(epilogue != GPT_EPI_BIAS_RESIDUAL, "gpt_gemm_fused: LayerNorm fold with a residual epilogue");
  } else if (!f.ln_sums) {
    GPT_CHECK_ARG(epilogue == GPT_EPI_NONE || bias, "gpt_gemm_fused: epilogue needs bias");
  }
  if (f.k_cache || f.v_cache) {
    GPT_CHECK_ARG(f.k_cache && f.v_cache && f.kv_heads > 0 && f.kv_dim > 0 && f.kv_tmax > 0 && f.kv_pos0 >= 0,
                  "gpt_gemm_fused: incomplete KV append");
    GPT_CHECK_SHAPE(N == 3 * f.kv_heads * f.kv_dim, "gpt_gemm_fused: KV append needs N = 3 * heads * dim");
  }
  GPT_CHECK_ARG(!(f.ln_stats && f.ln_sums), "gpt_gemm_fused: give ln_stats or ln_sums, not both");
  if (f.ln_sums)
    GPT_CHECK_ARG(f.ln_u && f.ln_v && f.ln_eps >= 0.f && epilogue != GPT_EPI_BIAS_RESIDUAL,
                  "gpt_gemm_fused: incomplete LayerNorm fold");
  GPT_CHECK_ARG(gpt::tc::tc_eligible(A, lda, W, K, M, N),
                "gpt_gemm_fused: operands must be 16-byte aligned with 16-byte row pitches");
  // Exact fp64 row sums (and, with them, the KV append) run on the 16-column decode GEMM.
  if (f.row_sums || (f.ln_sums && gpt::tc::rows_eligible(A, lda, W, C, ldc, M, N, K))) {
    GPT_CHECK_ARG(!f.ln_stats && !f.row_stats, "gpt_gemm_fused: fp32 parts and fp64 sums cannot be mixed");
    GPT_CHECK_SHAPE(gpt::tc::rows_eligible(A, lda, W, C, ldc, M, N, K),
                    "gpt_gemm_fused: row_sums need M <= 128 and N %% 16 == 0 (M=%lld N=%lld)", (long long)M,
                    (long long)N);
    return gpt::tc::gemm_rows(A, lda, W, bias, R, ldr, C, ldc, M, N, K, epilogue, &f, (cudaStream_t)stream);
  }
  GPT_CHECK_ARG(!f.ln_sums || M <= gpt::tc::kSkMaxM, "gpt_gemm_fused: ln_sums serve at most %d rows",
                gpt::tc::kSkMaxM);
  if (M <= gpt::tc::kSkMaxM)
    return gpt::tc::gemm_skinny_fused(A, lda, W, bias, R, ldr, C, ldc, M, N, K, epilogue, f, (cudaStream_t)stream);
  // more rows (prefill): the tcgen05 GEMM with the LayerNorm fold or row statistics
  GPT_CHECK_ARG(!f.k_cache, "gpt_gemm_fused: the KV append is a decode extra (M <= %d)", gpt::tc::kSkMaxM);
  return gpt::tc::gemm_bf16(A, lda, W, bias, R, ldr, C, ldc, M, N, K, epilogue, (cudaStream_t)stream, &f);
}

