// Causal prefill attention (flash-style online softmax, exp2 domain), the
// counterpart of causal_attention_kernel (cutile_gpt/kernels/attention.py:24-116).
//
//   attn_simt_kernel  fp32 (or bf16) I/O, any head_dim <= 128: one thread per
//                     query, K/V tiles staged in shared memory (broadcast
//                     reads), fp32 throughout. Serves the fp32 configs.
//   attn_mma_kernel   bf16, head_dim 64: 64-query x 64-key tiles, 4 warps,
//                     tensor-core QKᵀ and PV, cp.async double-buffered K/V,
//                     XOR-swizzled shared memory for ldmatrix.
// Both read q/k/v through (b, h, t) strides so they consume the fused QKV
// GEMM output [B, T, 3C] directly and write [B, T, C] for c_proj, removing
// the split / transpose / contiguous copies of cutile_gpt/models/gpt.py:133-146.
#include <stdlib.h>

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

// ---------------------------------------------------------------------------
// bf16 tensor-core kernel, head_dim 64.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  int n = pred ? 16 : 0;  // src-size 0 -> zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N_>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N_) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

constexpr int kBM = 64, kBN = 64, kD = 64;
// Byte offset of (row, col) in a [64][64] bf16 tile with 16-byte chunks
// XOR-swizzled by row (conflict-free ldmatrix and cp.async).
__device__ __forceinline__ uint32_t swz(int row, int col) {
  return (uint32_t)(row * 128 + ((((col >> 3) ^ (row & 7)) << 4)) + (col & 7) * 2);
}

__global__ void __launch_bounds__(128) attn_mma_kernel(const __nv_bfloat16* __restrict__ q,
                                                       const __nv_bfloat16* __restrict__ k,
                                                       const __nv_bfloat16* __restrict__ v,
                                                       __nv_bfloat16* __restrict__ o, Strides qs,
                                                       Strides ks, Strides vs, Strides os, int H, int T_,
                                                       float scale_log2) {
  pdl_wait();
  pdl_trigger();
  __shared__ __align__(128) uint8_t sQ[kBM * kD * 2];
  __shared__ __align__(128) uint8_t sK[2][kBN * kD * 2];
  __shared__ __align__(128) uint8_t sV[2][kBN * kD * 2];
  const int nqb = (T_ + kBM - 1) / kBM;
  const int qb = nqb - 1 - blockIdx.x;  // heaviest (longest causal span) blocks first
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = qb * kBM;
  const __nv_bfloat16* qbase = q + b * qs.b + h * qs.h;
  const __nv_bfloat16* kbase = k + b * ks.b + h * ks.h;
  const __nv_bfloat16* vbase = v + b * vs.b + h * vs.h;
  const uint32_t sQa = (uint32_t)__cvta_generic_to_shared(sQ);
  const uint32_t sKa[2] = {(uint32_t)__cvta_generic_to_shared(sK[0]), (uint32_t)__cvta_generic_to_shared(sK[1])};
  const uint32_t sVa[2] = {(uint32_t)__cvta_generic_to_shared(sV[0]), (uint32_t)__cvta_generic_to_shared(sV[1])};

  // Each thread moves 4 of the 512 16-byte chunks of a 64x64 tile.
  auto load_tile = [&](uint32_t dst, const __nv_bfloat16* src, int64_t st, int r0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int c = tid + i * 128;
      int row = c >> 3, ch = c & 7;
      bool ok = r0 + row < T_;
      const __nv_bfloat16* g = src + (int64_t)(ok ? r0 + row : 0) * st + ch * 8;
      cp_async16(dst + swz(row, ch * 8), g, ok);
    }
  };
  load_tile(sQa, qbase, qs.t, q0);
  load_tile(sKa[0], kbase, ks.t, 0);
  load_tile(sVa[0], vbase, vs.t, 0);
  cp_async_commit();

  float oacc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) oacc[i][j] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  uint32_t qf[4][4];
  const int nkb = qb + 1;  // causal: key blocks 0..qb
  const int g = lane >> 2, tig = lane & 3;
  const int qrow0 = q0 + warp * 16 + g;  // rows qrow0 and qrow0 + 8

  for (int j = 0; j < nkb; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkb) {
      load_tile(sKa[buf ^ 1], kbase, ks.t, (j + 1) * kBN);
      load_tile(sVa[buf ^ 1], vbase, vs.t, (j + 1) * kBN);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        int row = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        int col = kk * 16 + 8 * (lane >> 4);
        ldsm_x4(sQa + swz(row, col), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    // S = Q Kᵀ  (16 x 64 per warp)
    float s[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int i = 0; i < 4; ++i) s[nb][i] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int nb = 0; nb < 8; nb += 2) {
        uint32_t b0, b1, b2, b3;
        int key = 8 * (nb + (lane >> 4)) + (lane & 7);
        int col = kk * 16 + 8 * ((lane >> 3) & 1);
        ldsm_x4(sKa[buf] + swz(key, col), b0, b1, b2, b3);
        mma_bf16(s[nb], qf[kk], b0, b1);
        mma_bf16(s[nb + 1], qf[kk], b2, b3);
      }
    }
    // scale, causal / length mask, online softmax
    const int key0 = j * kBN;
    float mnew[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        int row = qrow0 + (i >> 1) * 8;
        int key = key0 + nb * 8 + tig * 2 + (i & 1);
        float x = s[nb][i] * scale_log2;
        if (key > row || key >= T_) x = -INFINITY;
        s[nb][i] = x;
        mnew[i >> 1] = fmaxf(mnew[i >> 1], x);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mnew[r] = fmaxf(mnew[r], __shfl_xor_sync(0xffffffffu, mnew[r], 1));
      mnew[r] = fmaxf(mnew[r], __shfl_xor_sync(0xffffffffu, mnew[r], 2));
      // A row with no valid key so far keeps m = -inf; use 0 as the shift.
      float mref = mnew[r] == -INFINITY ? 0.f : mnew[r];
      alpha[r] = exp2f(mrow[r] - mref);
      mrow[r] = mnew[r];
      mnew[r] = mref;
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pf[4][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      float p0 = exp2f(s[nb][0] - mnew[0]);
      float p1 = exp2f(s[nb][1] - mnew[0]);
      float p2 = exp2f(s[nb][2] - mnew[1]);
      float p3 = exp2f(s[nb][3] - mnew[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      // C fragment of n-block nb -> half of the A fragment of k-step nb/2.
      pf[nb >> 1][(nb & 1) * 2 + 0] = pack_bf16(p0, p1);
      pf[nb >> 1][(nb & 1) * 2 + 1] = pack_bf16(p2, p3);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) lrow[r] = lrow[r] * alpha[r] + rs[r];
#pragma unroll
    for (int db = 0; db < 8; ++db) {
      oacc[db][0] *= alpha[0];
      oacc[db][1] *= alpha[0];
      oacc[db][2] *= alpha[1];
      oacc[db][3] *= alpha[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int db = 0; db < 8; db += 2) {
        uint32_t b0, b1, b2, b3;
        int key = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        int col = 8 * (db + (lane >> 4));
        ldsm_x4_t(sVa[buf] + swz(key, col), b0, b1, b2, b3);
        mma_bf16(oacc[db], pf[kk], b0, b1);
        mma_bf16(oacc[db + 1], pf[kk], b2, b3);
      }
    }
    __syncthreads();  // buffer `buf` is refilled next iteration
  }
  // finalize: full row sums across the quad, normalise, store bf16 pairs
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  __nv_bfloat16* obase = o + b * os.b + h * os.h;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    int row = qrow0 + r * 8;
    if (row >= T_) continue;
    float inv = 1.f / lrow[r];
    __nv_bfloat16* orow = obase + (int64_t)row * os.t;
#pragma unroll
    for (int db = 0; db < 8; ++db) {
      int col = db * 8 + tig * 2;
      *reinterpret_cast<uint32_t*>(orow + col) = pack_bf16(oacc[db][r * 2] * inv, oacc[db][r * 2 + 1] * inv);
    }
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
    // GPT_ATTN_IMPL=mma selects the mma.sync kernel (comparison runs).
    static const bool force_mma = [] {
      const char* e = getenv("GPT_ATTN_IMPL");
      return e && e[0] == 'm';
    }();
    if (!force_mma && gpt::attn_tc::eligible(D, q, k, v, out, q_strides, k_strides, v_strides, o_strides))
      return gpt::attn_tc::launch(q, k, v, out, B, H, T, q_strides, k_strides, v_strides, o_strides, sl2, st);
    auto al = [](const void* p, int64_t s1, int64_t s2, int64_t s3) {
      return gpt::aligned(p, 16) && (s1 % 8) == 0 && (s2 % 8) == 0 && (s3 % 8) == 0;
    };
    if (D == 64 && al(q, qs.b, qs.h, qs.t) && al(k, ks.b, ks.h, ks.t) && al(v, vs.b, vs.h, vs.t) &&
        gpt::aligned(out, 4) && os.b % 2 == 0 && os.h % 2 == 0 && os.t % 2 == 0) {
      dim3 grid((unsigned)((T + kBM - 1) / kBM), (unsigned)(B * H));
      gpt::launch_pdl(attn_mma_kernel, dim3(grid), dim3(128), 0, st, (const __nv_bfloat16*)q, (const __nv_bfloat16*)k,
                                            (const __nv_bfloat16*)v, (__nv_bfloat16*)out, qs, ks, vs, os,
                                            (int)H, (int)T, sl2);
      return gpt::launch_status("attention_mma");
    }
    return launch_simt<__nv_bfloat16>(q, k, v, out, qs, ks, vs, os, B, H, T, D, sl2, st);
  }
  return launch_simt<float>(q, k, v, out, qs, ks, vs, os, B, H, T, D, sl2, st);
}
