// HBM-bound kernels: token+position embedding gather, LayerNorm, tanh-GELU,
// KV-cache append and the greedy argmax. All are written for 128-bit
// (16-byte) vector accesses with a scalar tail/fallback for unaligned data.
#include "common.cuh"

namespace gpt {

template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};

// Loads/stores 16 bytes as N floats.
template <typename T>
__device__ __forceinline__ void load16(const T* p, float* out) {
  uint4 raw = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec16<T>::N; ++i) out[i] = Tr<T>::to_f(e[i]);
}
template <typename T>
__device__ __forceinline__ void store16(T* p, const float* in) {
  uint4 raw;
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec16<T>::N; ++i) e[i] = Tr<T>::from_f(in[i]);
  *reinterpret_cast<uint4*>(p) = raw;
}

// ============================================================================
// Embedding: out[i] = wte[idx[i]] (+ wpe[pos0 + i % T]).  One warp per token
// row; 16-byte vectors when C is a multiple of the vector width.
// cutile_gpt/kernels/embedding.py:23-51 (gather) and cutile_gpt/models/gpt.py:110-113
// (token + position add) in one pass.
// ============================================================================
template <typename T, bool kPos, bool kVec>
__global__ void embedding_kernel(const int64_t* __restrict__ idx, int64_t n_tok,
                                 const T* __restrict__ wte, const T* __restrict__ wpe,
                                 int64_t vocab, int64_t n_pos, int64_t C, int64_t T_,
                                 int64_t pos0, const int64_t* __restrict__ pos_dev,
                                 T* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  int warps = blockDim.x >> 5;
  int64_t tok = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (tok >= n_tok) return;
  int64_t id = idx[tok];
  int64_t pos = kPos ? pos0 + (pos_dev ? *pos_dev : 0) + (tok % T_) : 0;
  bool ok = id >= 0 && id < vocab && (!kPos || (pos >= 0 && pos < n_pos));
  if (!ok && lane == 0) record_device_error(GPT_DEVERR_INDEX);
  const T* src = wte + (ok ? id : 0) * C;
  const T* psrc = kPos ? wpe + (ok ? pos : 0) * C : nullptr;
  T* dst = out + tok * C;
  if (kVec) {
    constexpr int V = Vec16<T>::N;
    for (int64_t c = (int64_t)lane * V; c < C; c += 32 * V) {
      float a[V];
      load16(src + c, a);
      if (kPos) {
        float b[V];
        load16(psrc + c, b);
#pragma unroll
        for (int i = 0; i < V; ++i) a[i] += b[i];
      }
      if (!ok) {
#pragma unroll
        for (int i = 0; i < V; ++i) a[i] = 0.f;
      }
      store16(dst + c, a);
    }
  } else {
    for (int64_t c = lane; c < C; c += 32) {
      float a = Tr<T>::to_f(src[c]);
      if (kPos) a += Tr<T>::to_f(psrc[c]);
      dst[c] = Tr<T>::from_f(ok ? a : 0.f);
    }
  }
}

template <typename T>
static int launch_embedding(const int64_t* idx, int64_t n_tok, const void* wte, const void* wpe,
                            int64_t vocab, int64_t n_pos, int64_t C, int64_t T_, int64_t pos0,
                            const int64_t* pos_dev, void* out, cudaStream_t st) {
  constexpr int V = Vec16<T>::N;
  bool vec = (C % V == 0) && aligned(wte, 16) && aligned(out, 16) && (!wpe || aligned(wpe, 16));
  const int warps = 4;
  dim3 grid((unsigned)((n_tok + warps - 1) / warps));
  const T* a = (const T*)wte;
  const T* b = (const T*)wpe;
  T* o = (T*)out;
  if (wpe) {
    if (vec) launch_pdl(embedding_kernel<T, true, true>, dim3(grid), dim3(warps * 32), 0, st, idx, n_tok, a, b, vocab, n_pos, C, T_, pos0, pos_dev, o);
    else launch_pdl(embedding_kernel<T, true, false>, dim3(grid), dim3(warps * 32), 0, st, idx, n_tok, a, b, vocab, n_pos, C, T_, pos0, pos_dev, o);
  } else {
    if (vec) launch_pdl(embedding_kernel<T, false, true>, dim3(grid), dim3(warps * 32), 0, st, idx, n_tok, a, b, vocab, n_pos, C, 1, 0, nullptr, o);
    else launch_pdl(embedding_kernel<T, false, false>, dim3(grid), dim3(warps * 32), 0, st, idx, n_tok, a, b, vocab, n_pos, C, 1, 0, nullptr, o);
  }
  return launch_status("embedding");
}

// ============================================================================
// LayerNorm: one warp per row, row cached in registers (up to NV 16-byte
// vectors per lane), exact two-pass statistics in fp32:
//   mean = sum(x)/C, var = sum((x-mean)^2)/C, y = (x-mean)*rsqrt(var+eps)*w+b.
// The reference kernel (cutile_gpt/kernels/layernorm.py:58-62) forms
// var = E[x^2] - mean^2; its CuPy oracle (layernorm.py:139-149) uses the
// two-pass form, which is what is computed here (same value in exact
// arithmetic, no cancellation).
// ============================================================================
template <typename T, int NV>
__global__ void __launch_bounds__(128) layernorm_vec_kernel(const T* __restrict__ x,
                                                            const T* __restrict__ w,
                                                            const T* __restrict__ b, T* y,
                                                            int64_t M, int C, float eps) {
  pdl_wait();
  pdl_trigger();
  constexpr int V = Vec16<T>::N;
  int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (row >= M) return;
  const T* xr = x + row * C;
  float v[NV][V];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    int c = (i * 32 + lane) * V;
    if (c < C) {
      load16(xr + c, v[i]);
#pragma unroll
      for (int j = 0; j < V; ++j) s += v[i][j];
    }
  }
  float mean = warp_sum(s) / (float)C;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    int c = (i * 32 + lane) * V;
    if (c < C) {
#pragma unroll
      for (int j = 0; j < V; ++j) {
        float d = v[i][j] - mean;
        q += d * d;
      }
    }
  }
  float rstd = rsqrtf(warp_sum(q) / (float)C + eps);
  T* yr = y + row * C;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    int c = (i * 32 + lane) * V;
    if (c < C) {
      float wv[V], bv[V], o[V];
      load16(w + c, wv);
      load16(b + c, bv);
#pragma unroll
      for (int j = 0; j < V; ++j) o[j] = (v[i][j] - mean) * rstd * wv[j] + bv[j];
      store16(yr + c, o);
    }
  }
}

// Any C, any alignment: one warp per row, three passes over the row (the
// second and third hit L1).
template <typename T>
__global__ void __launch_bounds__(128) layernorm_generic_kernel(const T* __restrict__ x,
                                                                const T* __restrict__ w,
                                                                const T* __restrict__ b, T* y,
                                                                int64_t M, int C, float eps) {
  pdl_wait();
  pdl_trigger();
  int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (row >= M) return;
  const T* xr = x + row * C;
  float s = 0.f;
  for (int c = lane; c < C; c += 32) s += Tr<T>::to_f(xr[c]);
  float mean = warp_sum(s) / (float)C;
  float q = 0.f;
  for (int c = lane; c < C; c += 32) {
    float d = Tr<T>::to_f(xr[c]) - mean;
    q += d * d;
  }
  float rstd = rsqrtf(warp_sum(q) / (float)C + eps);
  T* yr = y + row * C;
  for (int c = lane; c < C; c += 32) {
    float o = (Tr<T>::to_f(xr[c]) - mean) * rstd * Tr<T>::to_f(w[c]) + Tr<T>::to_f(b[c]);
    yr[c] = Tr<T>::from_f(o);
  }
}

template <typename T>
static int launch_layernorm(const void* x, const void* w, const void* b, void* y, int64_t M,
                            int64_t C, float eps, cudaStream_t st) {
  constexpr int V = Vec16<T>::N;
  dim3 grid((unsigned)((M + 3) / 4));
  const T *xp = (const T*)x, *wp = (const T*)w, *bp = (const T*)b;
  T* yp = (T*)y;
  bool vec = (C % V == 0) && aligned(x, 16) && aligned(w, 16) && aligned(b, 16) && aligned(y, 16);
  int nv = (int)((C + 32 * V - 1) / (32 * V));
  if (vec && nv <= 8) {
    switch (nv) {
#define GPT_LN_CASE(n) \
  case n: launch_pdl(layernorm_vec_kernel<T, n>, dim3(grid), dim3(128), 0, st, xp, wp, bp, yp, M, (int)C, eps); break;
      GPT_LN_CASE(1) GPT_LN_CASE(2) GPT_LN_CASE(3) GPT_LN_CASE(4)
      GPT_LN_CASE(5) GPT_LN_CASE(6) GPT_LN_CASE(7) GPT_LN_CASE(8)
#undef GPT_LN_CASE
      default: break;
    }
  } else {
    launch_pdl(layernorm_generic_kernel<T>, dim3(grid), dim3(128), 0, st, xp, wp, bp, yp, M, (int)C, eps);
  }
  return launch_status("layernorm");
}

// ============================================================================
// tanh-GELU, elementwise. Grid sized to a multiple of the SM count
// (grid-stride loop), 16-byte vectors + scalar tail.
// cutile_gpt/kernels/gelu.py:20-41.
// ============================================================================
template <typename T, bool kFast>
__global__ void __launch_bounds__(256) gelu_kernel(const T* x, T* y, int64_t n) {
  pdl_wait();
  pdl_trigger();
  constexpr int V = Vec16<T>::N;
  int64_t nvec = n / V;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    float a[V];
    load16(x + i * V, a);
#pragma unroll
    for (int j = 0; j < V; ++j) a[j] = gelu_tanh<kFast>(a[j]);
    store16(y + i * V, a);
  }
  for (int64_t i = nvec * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = Tr<T>::from_f(gelu_tanh<kFast>(Tr<T>::to_f(x[i])));
}

template <typename T, bool kFast>
__global__ void __launch_bounds__(256) gelu_scalar_kernel(const T* x, T* y, int64_t n) {
  pdl_wait();
  pdl_trigger();
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = Tr<T>::from_f(gelu_tanh<kFast>(Tr<T>::to_f(x[i])));
}

template <typename T, bool kFast>
static int launch_gelu(const void* x, void* y, int64_t n, cudaStream_t st) {
  constexpr int V = Vec16<T>::N;
  int sms = device_sm_count();
  if (sms <= 0) sms = 148;
  int64_t work = (n + V - 1) / V;
  int64_t blocks = (work + 255) / 256;
  int64_t cap = (int64_t)sms * 8;  // 8 resident 256-thread CTAs per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (aligned(x, 16) && aligned(y, 16))
    launch_pdl(gelu_kernel<T, kFast>, dim3((unsigned)blocks), dim3(256), 0, st, (const T*)x, (T*)y, n);
  else
    launch_pdl(gelu_scalar_kernel<T, kFast>, dim3((unsigned)blocks), dim3(256), 0, st, (const T*)x, (T*)y, n);
  return launch_status("gelu");
}

// ============================================================================
// KV append: k/v of Tn new positions from the QKV buffer [B, Tn, 3C] into
// the caches [B, H, Tmax, D] at pos0.. One thread per 16-byte vector.
// ============================================================================
template <typename T>
__global__ void kv_append_kernel(const T* __restrict__ qkv, int64_t ld, T* __restrict__ kc,
                                 T* __restrict__ vc, int64_t B, int64_t H, int64_t Tn, int64_t D,
                                 int64_t Tmax, int64_t pos0, const int64_t* __restrict__ pos_dev) {
  pdl_wait();
  pdl_trigger();
  constexpr int V = Vec16<T>::N;
  int64_t C = H * D;
  if (pos_dev) pos0 += *pos_dev;
  int64_t dv = D / V;
  int64_t total = B * Tn * H * dv;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t d = (i % dv) * V;
    int64_t h = (i / dv) % H;
    int64_t t = (i / (dv * H)) % Tn;
    int64_t b = i / (dv * H * Tn);
    const T* src = qkv + (b * Tn + t) * ld + h * D + d;
    if (pos0 + t < 0 || pos0 + t >= Tmax) {
      record_device_error(GPT_DEVERR_INDEX);
      continue;
    }
    int64_t off = ((b * H + h) * Tmax + pos0 + t) * D + d;
    *reinterpret_cast<uint4*>(kc + off) = *reinterpret_cast<const uint4*>(src + C);
    *reinterpret_cast<uint4*>(vc + off) = *reinterpret_cast<const uint4*>(src + 2 * C);
  }
}

// ============================================================================
// Greedy argmax per row (first index on ties), one CTA per row. A row is
// ~100 KB of logits: 1024 threads, each with 8 independent loads in flight
// before any compare, so the row streams at L2 bandwidth instead of one load
// latency per element.
// ============================================================================
constexpr int kArgmaxThreads = 1024;
template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const T* __restrict__ logits, int64_t ld,
                                                                int64_t V, int64_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const T* row = logits + (int64_t)blockIdx.x * ld;
  float best = -INFINITY;
  int64_t bi = V;  // sentinel larger than any index
  constexpr int kIlp = 8;
  for (int64_t base = 0; base < V; base += (int64_t)kIlp * blockDim.x) {
    float v[kIlp];
#pragma unroll
    for (int u = 0; u < kIlp; ++u) {
      const int64_t i = base + (int64_t)u * blockDim.x + threadIdx.x;
      v[u] = i < V ? Tr<T>::to_f(__ldg(row + i)) : __int_as_float(0x7fc00000);  // NaN never wins
    }
#pragma unroll
    for (int u = 0; u < kIlp; ++u) {
      const int64_t i = base + (int64_t)u * blockDim.x + threadIdx.x;
      // strictly larger wins (indices rise within a thread, so the first
      // index is kept); the first non-NaN value is taken even when it is
      // -inf. NaNs never win.
      if (v[u] > best || (bi == V && v[u] >= best)) { best = v[u]; bi = i; }
    }
  }
  // (value, index) reduction: larger value wins, smaller index on ties.
  __shared__ float sv[32];
  __shared__ int64_t si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[w] = best; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : V;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best, o);
      int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) out[blockIdx.x] = bi < V ? bi : 0;
  }
}

// End of a decode step: record the new tokens at column *pos + 1, then
// advance the device position. One CTA, so every thread reads *pos before
// thread 0 bumps it.
__global__ void decode_advance_kernel(const int64_t* __restrict__ tok, int64_t B, int64_t* seq,
                                      int64_t ld_seq, int64_t seq_len, int64_t* pos) {
  pdl_wait();
  pdl_trigger();
  const int64_t col = *pos + 1;
  if (seq && col >= 0 && col < seq_len)
    for (int64_t b = threadIdx.x; b < B; b += blockDim.x) seq[b * ld_seq + col] = tok[b];
  __syncthreads();
  if (threadIdx.x == 0) *pos = col;
}

// ============================================================================
// Row statistics (sum, sum of squares) of x [M, C]: the LayerNorm statistics
// a folded decode GEMM consumes (one part). One warp per row.
// ============================================================================
template <typename T>
__global__ void __launch_bounds__(256) row_stats_kernel(const T* __restrict__ x, int64_t ld, int64_t M, int64_t C,
                                                        float* __restrict__ stats) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const T* xr = x + row * ld;
  float s1 = 0.f, s2 = 0.f;
  for (int64_t i = lane; i < C; i += 32) {
    const float v = Tr<T>::to_f(xr[i]);
    s1 += v;
    s2 = fmaf(v, v, s2);
  }
  s1 = warp_sum(s1);
  s2 = warp_sum(s2);
  if (lane == 0) {
    stats[row * 2] = s1;
    stats[row * 2 + 1] = s2;
  }
}

// LayerNorm fold of a Linear that follows LayerNorm(gamma, beta): one warp
// per output row n. Wf[n, k] = W[n, k] * gamma[k] (rounded to T);
// u[n] = sum_k Wf[n, k]; v[n] = sum_k W[n, k] * beta[k] + bias[n].
template <typename T>
__global__ void __launch_bounds__(256) lnfold_kernel(const T* __restrict__ W, const T* __restrict__ gamma,
                                                     const T* __restrict__ beta, const T* __restrict__ bias,
                                                     int64_t N, int64_t K, T* __restrict__ Wf,
                                                     float* __restrict__ u, float* __restrict__ v) {
  pdl_wait();
  pdl_trigger();
  const int64_t n = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  float su = 0.f, sv = 0.f;
  for (int64_t k = lane; k < K; k += 32) {
    const float w = Tr<T>::to_f(W[n * K + k]);
    const T wf = Tr<T>::from_f(w * Tr<T>::to_f(gamma[k]));
    Wf[n * K + k] = wf;
    su += Tr<T>::to_f(wf);
    sv = fmaf(w, Tr<T>::to_f(beta[k]), sv);
  }
  su = warp_sum(su);
  sv = warp_sum(sv);
  if (lane == 0) {
    u[n] = su;
    v[n] = sv + (bias ? Tr<T>::to_f(bias[n]) : 0.f);
  }
}

}  // namespace gpt

// ============================================================================
// C ABI
// ============================================================================
extern "C" {

int gpt_embedding(const int64_t* idx, int64_t n_idx, const void* weight, int64_t vocab, int64_t C,
                  void* out, int dtype, void* stream) {
  GPT_CHECK_DTYPE(dtype);
  GPT_CHECK_SHAPE(n_idx >= 0 && vocab > 0 && C > 0, "gpt_embedding: bad sizes n=%lld vocab=%lld C=%lld",
                  (long long)n_idx, (long long)vocab, (long long)C);
  if (n_idx == 0) return GPT_OK;
  GPT_CHECK_ARG(idx && weight && out, "gpt_embedding: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == GPT_F32)
    return gpt::launch_embedding<float>(idx, n_idx, weight, nullptr, vocab, 0, C, 1, 0, nullptr, out, st);
  return gpt::launch_embedding<__nv_bfloat16>(idx, n_idx, weight, nullptr, vocab, 0, C, 1, 0, nullptr, out, st);
}

int gpt_embedding_pos(const int64_t* idx, int64_t B, int64_t T, const void* wte, const void* wpe,
                      int64_t vocab, int64_t n_pos, int64_t C, int64_t pos0, const int64_t* pos_dev,
                      void* out, int dtype, void* stream) {
  GPT_CHECK_DTYPE(dtype);
  GPT_CHECK_SHAPE(B >= 0 && T >= 0 && vocab > 0 && C > 0 && n_pos > 0 && pos0 >= 0 &&
                      (pos_dev != nullptr || pos0 + T <= n_pos),
                  "gpt_embedding_pos: bad sizes B=%lld T=%lld pos0=%lld n_pos=%lld", (long long)B,
                  (long long)T, (long long)pos0, (long long)n_pos);
  if (B * T == 0) return GPT_OK;
  GPT_CHECK_ARG(idx && wte && wpe && out, "gpt_embedding_pos: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == GPT_F32)
    return gpt::launch_embedding<float>(idx, B * T, wte, wpe, vocab, n_pos, C, T, pos0, pos_dev, out, st);
  return gpt::launch_embedding<__nv_bfloat16>(idx, B * T, wte, wpe, vocab, n_pos, C, T, pos0, pos_dev, out, st);
}

int gpt_layernorm(const void* x, const void* w, const void* b, void* y, int64_t M, int64_t C, float eps,
                  int dtype, void* stream) {
  GPT_CHECK_DTYPE(dtype);
  GPT_CHECK_SHAPE(M >= 0 && C > 0 && C <= (1 << 24), "gpt_layernorm: bad sizes M=%lld C=%lld",
                  (long long)M, (long long)C);
  if (M == 0) return GPT_OK;
  GPT_CHECK_ARG(x && w && b && y, "gpt_layernorm: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == GPT_F32) return gpt::launch_layernorm<float>(x, w, b, y, M, C, eps, st);
  return gpt::launch_layernorm<__nv_bfloat16>(x, w, b, y, M, C, eps, st);
}

int gpt_gelu(const void* x, void* y, int64_t n, int dtype, void* stream) {
  GPT_CHECK_DTYPE(dtype);
  GPT_CHECK_SHAPE(n >= 0, "gpt_gelu: negative size");
  if (n == 0) return GPT_OK;
  GPT_CHECK_ARG(x && y, "gpt_gelu: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == GPT_F32) return gpt::launch_gelu<float, false>(x, y, n, st);
  return gpt::launch_gelu<__nv_bfloat16, true>(x, y, n, st);
}

int gpt_kv_append(const void* qkv, int64_t ld_qkv, void* k_cache, void* v_cache, int64_t B, int64_t H,
                  int64_t Tn, int64_t D, int64_t Tmax, int64_t pos0, const int64_t* pos_dev, int dtype,
                  void* stream) {
  GPT_CHECK_DTYPE(dtype);
  GPT_CHECK_SHAPE(B >= 0 && H > 0 && Tn >= 0 && D > 0 && pos0 >= 0 && (pos_dev || pos0 + Tn <= Tmax) &&
                      ld_qkv >= 3 * H * D,
                  "gpt_kv_append: bad sizes B=%lld H=%lld Tn=%lld D=%lld Tmax=%lld pos0=%lld",
                  (long long)B, (long long)H, (long long)Tn, (long long)D, (long long)Tmax,
                  (long long)pos0);
  if (B * Tn == 0) return GPT_OK;
  GPT_CHECK_ARG(qkv && k_cache && v_cache, "gpt_kv_append: null pointer");
  size_t es = dtype == GPT_F32 ? 4 : 2;
  GPT_CHECK_ALIGN((D * es) % 16 == 0 && (ld_qkv * es) % 16 == 0 && gpt::aligned(qkv, 16) &&
                      gpt::aligned(k_cache, 16) && gpt::aligned(v_cache, 16),
                  "gpt_kv_append: needs 16-byte aligned rows");
  cudaStream_t st = (cudaStream_t)stream;
  int64_t vecs = B * Tn * H * (D * (int64_t)es / 16);
  int64_t blocks = (vecs + 255) / 256;
  if (blocks > 65535) blocks = 65535;
  if (dtype == GPT_F32)
    gpt::launch_pdl(gpt::kv_append_kernel<float>, dim3((unsigned)blocks), dim3(256), 0, st, 
        (const float*)qkv, ld_qkv, (float*)k_cache, (float*)v_cache, B, H, Tn, D, Tmax, pos0, pos_dev);
  else
    gpt::launch_pdl(gpt::kv_append_kernel<__nv_bfloat16>, dim3((unsigned)blocks), dim3(256), 0, st, 
        (const __nv_bfloat16*)qkv, ld_qkv, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, B, H, Tn,
        D, Tmax, pos0, pos_dev);
  return gpt::launch_status("kv_append");
}

int gpt_argmax(const void* logits, int64_t ld, int64_t B, int64_t V, int64_t* out, int dtype,
               void* stream) {
  GPT_CHECK_DTYPE(dtype);
  GPT_CHECK_SHAPE(B >= 0 && V > 0 && ld >= V && B < (1LL << 31), "gpt_argmax: bad sizes");
  if (B == 0) return GPT_OK;
  GPT_CHECK_ARG(logits && out, "gpt_argmax: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == GPT_F32)
    gpt::launch_pdl(gpt::argmax_kernel<float>, dim3((unsigned)B), dim3(gpt::kArgmaxThreads), 0, st, (const float*)logits, ld, V, out);
  else
    gpt::launch_pdl(gpt::argmax_kernel<__nv_bfloat16>, dim3((unsigned)B), dim3(gpt::kArgmaxThreads), 0, st, (const __nv_bfloat16*)logits, ld, V, out);
  return gpt::launch_status("argmax");
}

int gpt_decode_advance(const int64_t* tok, int64_t B, int64_t* seq, int64_t ld_seq, int64_t seq_len,
                       int64_t* pos_dev, void* stream) {
  GPT_CHECK_SHAPE(B >= 0 && (!seq || (ld_seq >= seq_len && seq_len >= 0)), "gpt_decode_advance: bad sizes");
  GPT_CHECK_ARG(pos_dev && (B == 0 || tok), "gpt_decode_advance: null pointer");
  gpt::launch_pdl(gpt::decode_advance_kernel, dim3(1), dim3(256), 0, (cudaStream_t)stream, tok, B, seq, ld_seq, seq_len, pos_dev);
  return gpt::launch_status("decode_advance");
}

int gpt_row_stats(const void* x, int64_t ld, int64_t M, int64_t C, float* stats, int dtype, void* stream) {
  GPT_CHECK_DTYPE(dtype);
  GPT_CHECK_SHAPE(M >= 0 && C > 0 && ld >= C, "gpt_row_stats: bad sizes");
  if (M == 0) return GPT_OK;
  GPT_CHECK_ARG(x && stats, "gpt_row_stats: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid((unsigned)((M + 7) / 8));
  if (dtype == GPT_F32)
    gpt::launch_pdl(gpt::row_stats_kernel<float>, grid, dim3(256), 0, st, (const float*)x, ld, M, C, stats);
  else
    gpt::launch_pdl(gpt::row_stats_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, (const __nv_bfloat16*)x, ld, M,
                    C, stats);
  return gpt::launch_status("row_stats");
}

int gpt_lnfold_weights(const void* W, const void* gamma, const void* beta, const void* bias, int64_t N, int64_t K,
                       void* Wf, float* u, float* v, int dtype, void* stream) {
  GPT_CHECK_DTYPE(dtype);
  GPT_CHECK_SHAPE(N >= 0 && K > 0, "gpt_lnfold_weights: bad sizes");
  if (N == 0) return GPT_OK;
  GPT_CHECK_ARG(W && gamma && beta && Wf && u && v, "gpt_lnfold_weights: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid((unsigned)((N + 7) / 8));
  if (dtype == GPT_F32)
    gpt::launch_pdl(gpt::lnfold_kernel<float>, grid, dim3(256), 0, st, (const float*)W, (const float*)gamma,
                    (const float*)beta, (const float*)bias, N, K, (float*)Wf, u, v);
  else
    gpt::launch_pdl(gpt::lnfold_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, (const __nv_bfloat16*)W,
                    (const __nv_bfloat16*)gamma, (const __nv_bfloat16*)beta, (const __nv_bfloat16*)bias, N, K,
                    (__nv_bfloat16*)Wf, u, v);
  return gpt::launch_status("lnfold_weights");
}

}  // extern "C"
