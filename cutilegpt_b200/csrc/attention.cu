// Causal prefill attention (flash-style online softmax, exp2 domain), the
// counterpart of causal_attention_kernel (cutile_gpt/kernels/attention.py:24-116).
//
//   attn_simt_kernel  fp32 (or bf16) I/O, any head_dim <= 128: one thread per
//                     query, K/V tiles staged in shared memory (broadcast
//                     reads), fp32 throughout. Serves the fp32 configs.
// bf16 with head_dim 64 and 16-byte aligned rows runs on the tcgen05 kernel
// (attention_tc.cu); every other request runs here. Both read q/k/v through (b, h, t) strides so they consume the fused QKV
// GEMM output [B, T, 3C] directly and write [B, T, C] for c_proj, removing
// the split / transpose / contiguous copies of cutile_gpt/models/gpt.py:133-146.
#include "common.cuh"

namespace gpt {
namespace attn {

constexpr float kLog2e = 1.4426950408889634f;

struct Strides {
  int64_t b, h, t;
};

// ---------------------------------------------------------------------------
template <typename T, int DM, int TN>
__global__ void __launch_bounds__(128) attn_simt_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                        const T* __restrict__ v, T* __restrict__ o,
                                                        Strides qs, Strides ks, Strides vs, Strides os,
                                                        int H, int T_, int D, float scale_log2) {
  pdl_wait();
  pdl_trigger();
  __shared__ float Ks[TN][DM];
  __shared__ float Vs[TN][DM];
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int q0 = blockIdx.x * 128;
  const int qi = q0 + threadIdx.x;
  const bool active = qi < T_;
  float qr[DM], acc[DM];
  const T* qp = q + b * qs.b + h * qs.h + (int64_t)qi * qs.t;
#pragma unroll
  for (int d = 0; d < DM; ++d) {
    qr[d] = (active && d < D) ? Tr<T>::to_f(qp[d]) * scale_log2 : 0.f;
    acc[d] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int kend = min(T_, q0 + 128);
  const T* kb = k + b * ks.b + h * ks.h;
  const T* vb = v + b * vs.b + h * vs.h;
  for (int k0 = 0; k0 < kend; k0 += TN) {
    for (int i = threadIdx.x; i < TN * DM; i += blockDim.x) {
      int j = i / DM, d = i % DM;
      int kj = k0 + j;
      bool ok = kj < kend && d < D;
      Ks[j][d] = ok ? Tr<T>::to_f(kb[(int64_t)kj * ks.t + d]) : 0.f;
      Vs[j][d] = ok ? Tr<T>::to_f(vb[(int64_t)kj * vs.t + d]) : 0.f;
    }
    __syncthreads();
    float s[TN];
    float mt = m;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      float dot = 0.f;
#pragma unroll
      for (int d = 0; d < DM; ++d) dot = fmaf(qr[d], Ks[j][d], dot);
      s[j] = (k0 + j <= qi && k0 + j < kend) ? dot : -INFINITY;
      mt = fmaxf(mt, s[j]);
    }
    if (mt != -INFINITY) {
      const float alpha = exp2f(m - mt);  // m = -inf -> 0
      l *= alpha;
#pragma unroll
      for (int d = 0; d < DM; ++d) acc[d] *= alpha;
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const float pj = exp2f(s[j] - mt);
        l += pj;
#pragma unroll
        for (int d = 0; d < DM; ++d) acc[d] = fmaf(pj, Vs[j][d], acc[d]);
      }
      m = mt;
    }
    __syncthreads();
  }
  if (active) {
    const float inv = 1.f / l;
    T* op = o + b * os.b + h * os.h + (int64_t)qi * os.t;
#pragma unroll
    for (int d = 0; d < DM; ++d)
      if (d < D) op[d] = Tr<T>::from_f(acc[d] * inv);
  }
}


template <typename T>
static int launch_simt(const void* q, const void* k, const void* v, void* o, Strides qs, Strides ks,
                       Strides vs, Strides os, int64_t B, int64_t H, int64_t T_, int64_t D, float sl2,
                       cudaStream_t st) {
  dim3 grid((unsigned)((T_ + 127) / 128), (unsigned)(B * H));
  const T *qq = (const T*)q, *kk = (const T*)k, *vv = (const T*)v;
  T* oo = (T*)o;
  if (D <= 16)
    launch_pdl(attn_simt_kernel<T, 16, 32>, dim3(grid), dim3(128), 0, st, qq, kk, vv, oo, qs, ks, vs, os, (int)H, (int)T_, (int)D, sl2);
  else if (D <= 32)
    launch_pdl(attn_simt_kernel<T, 32, 32>, dim3(grid), dim3(128), 0, st, qq, kk, vv, oo, qs, ks, vs, os, (int)H, (int)T_, (int)D, sl2);
  else if (D <= 64)
    launch_pdl(attn_simt_kernel<T, 64, 16>, dim3(grid), dim3(128), 0, st, qq, kk, vv, oo, qs, ks, vs, os, (int)H, (int)T_, (int)D, sl2);
  else
    launch_pdl(attn_simt_kernel<T, 128, 8>, dim3(grid), dim3(128), 0, st, qq, kk, vv, oo, qs, ks, vs, os, (int)H, (int)T_, (int)D, sl2);
  return launch_status("attention_simt");
}

}  // namespace attn
}  // namespace gpt

extern "C" int gpt_attention_prefill(const void* q, const void* k, const void* v, void* out, int64_t B,
                                     int64_t H, int64_t T, int64_t D, const int64_t* q_strides,
                                     const int64_t* k_strides, const int64_t* v_strides,
                                     const int64_t* o_strides, float scale, int dtype, void* stream) {
  using namespace gpt::attn;
  GPT_CHECK_DTYPE(dtype);
  GPT_CHECK_SHAPE(B >= 0 && H > 0 && T >= 0 && D > 0 && D <= 128 && B * H < 65536 && T < (1 << 30),
                  "gpt_attention_prefill: unsupported sizes B=%lld H=%lld T=%lld D=%lld", (long long)B,
                  (long long)H, (long long)T, (long long)D);
  if (B == 0 || T == 0) return GPT_OK;
  GPT_CHECK_ARG(q && k && v && out && q_strides && k_strides && v_strides && o_strides,
                "gpt_attention_prefill: null pointer");
  Strides qs{q_strides[0], q_strides[1], q_strides[2]}, ks{k_strides[0], k_strides[1], k_strides[2]},
      vs{v_strides[0], v_strides[1], v_strides[2]}, os{o_strides[0], o_strides[1], o_strides[2]};
  const float sl2 = scale * kLog2e;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == GPT_BF16) {
    if (gpt::attn_tc::eligible(D, q, k, v, out, q_strides, k_strides, v_strides, o_strides))
      return gpt::attn_tc::launch(q, k, v, out, B, H, T, q_strides, k_strides, v_strides, o_strides, sl2, st);
    return launch_simt<__nv_bfloat16>(q, k, v, out, qs, ks, vs, os, B, H, T, D, sl2, st);
  }
  return launch_simt<float>(q, k, v, out, qs, ks, vs, os, B, H, T, D, sl2, st);
}
