// One-query-per-(b, h) attention over the KV cache (decode step), split
// over the KV length (flash-decoding). No reference counterpart: the
// reference re-runs the whole prefix forward per generated token
// (cutile_gpt/models/gpt.py:204-206); with a KV cache each step reads the
// cached K/V once, which makes this kernel HBM-bound.
//
// Layout: caches [B, H, Tmax, D] (row = one position, D contiguous).
// A warp reads KPW keys per iteration, D*sizeof(T)/16 lanes per key, each
// lane one 16-byte vector, so one warp load instruction covers KPW whole
// K rows (512 B for bf16 D=64). Scores and the running (max, sum, acc)
// live in registers; warps and key groups are merged at the end.
#include "common.cuh"

namespace gpt {
namespace dec {

constexpr int kWarps = 4;
// Resident CTAs per SM the register budget must allow: the cfg-4 grid (64 x 12
// (b, h) pairs, one split) then runs as a single wave on 148 SMs instead of
// 1.04 waves at the 5 CTAs per SM that 92 registers per thread allow.
constexpr int kMinBlocks = 6;
constexpr float kLog2e = 1.4426950408889634f;

// Number of KV splits: enough CTAs to cover the SMs twice, at least 64
// positions per split, monotone non-decreasing in L (so a workspace sized
// for Tmax covers every step).
inline int num_splits(int64_t B, int64_t H, int64_t L, int sms) {
  int64_t bh = B * H;
  int64_t want = (2 * (int64_t)sms + bh - 1) / bh;
  int64_t cap = (L + 63) / 64;
  int64_t s = want < cap ? want : cap;
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  return (int)s;
}

template <typename T, int D>
__global__ void __launch_bounds__(kWarps * 32, kMinBlocks) decode_kernel(const T* __restrict__ q, int64_t ld_q,
                                                             const T* __restrict__ kc,
                                                             const T* __restrict__ vc, T* __restrict__ out,
                                                             int64_t ld_out, int H, int64_t Tmax, int L0,
                                                             const int64_t* __restrict__ len_dev,
                                                             float scale_log2, float* __restrict__ ws,
                                                             int prefetch) {
  // Before the dependency wait: start pulling this CTA's cached K/V rows
  // into L2. Rows below the current position were written by earlier steps,
  // so the reads overlap the tail of the preceding kernel (the QKV GEMM that
  // appends row L-1). A prefetch is only a hint: the length read here may be
  // stale without affecting results, and is clamped to the cache.
  if (prefetch) {
    int Lp = L0 + (len_dev ? (int)*reinterpret_cast<const volatile int64_t*>(len_dev) : 0);
    Lp = max(0, min(Lp, (int)Tmax));
    const int chunk = (Lp + gridDim.x - 1) / (int)gridDim.x;
    const int p0 = (int)blockIdx.x * chunk, p1 = min(Lp, p0 + chunk);
    constexpr int kPiece = 4096;   // bytes per prefetch instruction
    const int64_t bytes = p1 > p0 ? (int64_t)(p1 - p0) * D * (int64_t)sizeof(T) : 0;
    const int npieces = (int)((bytes + kPiece - 1) / kPiece);
    const int64_t row0 = ((int64_t)blockIdx.y * Tmax + p0) * D;
    for (int i = threadIdx.x; i < 2 * npieces; i += blockDim.x) {
      const T* src = ((i & 1) ? vc : kc) + row0;
      const int64_t off = (int64_t)(i >> 1) * kPiece;
      const int64_t rem = bytes - off;
      const uint32_t n = (uint32_t)(rem < kPiece ? rem : kPiece);   // whole rows: a multiple of 16 bytes
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<const char*>(src) + off),
                   "r"(n)
                   : "memory");
    }
  }
  pdl_wait();
  pdl_trigger();
  constexpr int V = 16 / sizeof(T);   // elements per lane vector
  constexpr int LPK = D / V;          // lanes per key
  constexpr int KPW = 32 / LPK;       // keys per warp iteration
  static_assert(D % V == 0 && 32 % LPK == 0, "unsupported head_dim");
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int split = blockIdx.x, nsplit = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane % LPK, grp = lane / LPK;
  int L = L0 + (len_dev ? (int)*len_dev : 0);
  if (L > Tmax) {
    if (threadIdx.x == 0 && split == 0) record_device_error(GPT_DEVERR_INDEX);
    L = (int)Tmax;
  }
  const int chunk = (L + nsplit - 1) / nsplit;
  const int c0 = split * chunk, c1 = min(L, c0 + chunk);

  float qv[V];
  {
    const T* qp = q + (int64_t)b * ld_q + (int64_t)h * D + sub * V;
    uint4 raw = *reinterpret_cast<const uint4*>(qp);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < V; ++i) qv[i] = Tr<T>::to_f(e[i]) * scale_log2;
  }
  const int64_t base = ((int64_t)b * H + h) * Tmax * D;
  const T* kb = kc + base + sub * V;
  const T* vb = vc + base + sub * V;
  float m = -INFINITY, l = 0.f, acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = 0.f;

  // kUnroll groups of KPW keys per warp step: every K and V vector of the
  // step is requested before the first dot product, so each lane keeps
  // 2 x kUnroll 16-byte loads in flight; the running max is updated once per
  // step.
  constexpr int kUnroll = 8;
  // Key group g (KPW keys) of the chunk belongs to warp g % kWarps, so the
  // warps of a CTA issue equal numbers of loads.
  for (int j0 = c0 + warp * KPW; j0 < c1; j0 += kWarps * KPW * kUnroll) {
    uint4 kr[kUnroll], vr[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int j = j0 + u * kWarps * KPW + grp;
      kr[u] = make_uint4(0, 0, 0, 0);
      vr[u] = make_uint4(0, 0, 0, 0);
      if (j < c1) {
        kr[u] = __ldcs(reinterpret_cast<const uint4*>(kb + (int64_t)j * D));
        vr[u] = __ldcs(reinterpret_cast<const uint4*>(vb + (int64_t)j * D));
      }
    }
    float dot[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const T* ke = reinterpret_cast<const T*>(&kr[u]);
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < V; ++i) d = fmaf(qv[i], Tr<T>::to_f(ke[i]), d);
      dot[u] = d;
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
#pragma unroll
      for (int o = 1; o < LPK; o <<= 1) dot[u] += __shfl_xor_sync(0xffffffffu, dot[u], o);
      if (j0 + u * kWarps * KPW + grp >= c1) dot[u] = -INFINITY;  // masked key
    }
    float mx = dot[0];
#pragma unroll
    for (int u = 1; u < kUnroll; ++u) mx = fmaxf(mx, dot[u]);
    const float mn = fmaxf(m, mx);
    if (mn != -INFINITY) {  // at least one live key in this lane's group
      const float a = exp2f(m - mn);
      l *= a;
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] *= a;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const float pu = exp2f(dot[u] - mn);  // 0 for a masked key
        l += pu;
        const T* ve = reinterpret_cast<const T*>(&vr[u]);
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = fmaf(pu, Tr<T>::to_f(ve[i]), acc[i]);
      }
      m = mn;
    }
  }
  // merge key groups inside the warp (lanes with equal `sub`)
#pragma unroll
  for (int o = LPK; o < 32; o <<= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, m, o);
    const float lo = __shfl_xor_sync(0xffffffffu, l, o);
    const float mn = fmaxf(m, mo);
    const float a = mn == -INFINITY ? 0.f : exp2f(m - mn);
    const float bo = mn == -INFINITY ? 0.f : exp2f(mo - mn);
    l = l * a + lo * bo;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float ao = __shfl_xor_sync(0xffffffffu, acc[i], o);
      acc[i] = acc[i] * a + ao * bo;
    }
    m = mn;
  }
  // merge warps through shared memory
  __shared__ float sm_m[kWarps], sm_l[kWarps];
  __shared__ float sm_acc[kWarps][D];
  if (grp == 0) {
#pragma unroll
    for (int i = 0; i < V; ++i) sm_acc[warp][sub * V + i] = acc[i];
    if (sub == 0) {
      sm_m[warp] = m;
      sm_l[warp] = l;
    }
  }
  __syncthreads();
  if (warp == 0) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm_m[w]);
    float Lsum = 0.f, wgt[kWarps];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      wgt[w] = M == -INFINITY ? 0.f : exp2f(sm_m[w] - M);
      Lsum += sm_l[w] * wgt[w];
    }
    for (int d = lane; d < D; d += 32) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) s += sm_acc[w][d] * wgt[w];
      if (nsplit == 1) {
        out[(int64_t)b * ld_out + (int64_t)h * D + d] = Tr<T>::from_f(s / Lsum);
      } else {
        float* part = ws + ((int64_t)bh * nsplit + split) * (D + 2);
        part[2 + d] = s;
        if (d == 0) {
          part[0] = M;
          part[1] = Lsum;
        }
      }
    }
  }
}

// Merges the per-split (max, sum, acc) partials. One CTA per (b, h), one
// thread per head dimension.
template <typename T, int D>
__global__ void combine_kernel(const float* __restrict__ ws, int nsplit, T* __restrict__ out, int64_t ld_out,
                               int H) {
  pdl_wait();
  pdl_trigger();
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int d = threadIdx.x;
  const float* part = ws + (int64_t)bh * nsplit * (D + 2);
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, part[s * (D + 2)]);
  float Ls = 0.f, acc = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float* p = part + s * (D + 2);
    const float w = p[0] == -INFINITY ? 0.f : exp2f(p[0] - M);
    Ls += p[1] * w;
    acc += p[2 + d] * w;
  }
  out[(int64_t)b * ld_out + (int64_t)h * D + d] = Tr<T>::from_f(acc / Ls);
}

template <typename T, int D>
static int launch(const void* q, int64_t ld_q, const void* kc, const void* vc, void* out, int64_t ld_out,
                  int64_t B, int64_t H, int64_t Tmax, int64_t L, const int64_t* len_dev, float sl2, void* ws,
                  cudaStream_t st) {
  int sms = device_sm_count();
  if (sms <= 0) sms = 148;
  int ns = num_splits(B, H, len_dev ? Tmax : L, sms);
  dim3 grid((unsigned)ns, (unsigned)(B * H));
  // The early L2 prefetch only pays while the launch's K/V fit comfortably in the 126 MB L2; a
  // larger cache (long contexts, big batches) would be evicted before its main loads and read twice.
  const int64_t kv_bytes = 2 * B * H * (len_dev ? Tmax : L) * (int64_t)D * (int64_t)sizeof(T);
  const int prefetch = kv_bytes <= (int64_t(64) << 20) ? 1 : 0;
  launch_pdl(decode_kernel<T, D>, dim3(grid), dim3(kWarps * 32), 0, st, (const T*)q, ld_q, (const T*)kc, (const T*)vc, (T*)out,
                                                    ld_out, (int)H, Tmax, (int)L, len_dev, sl2, (float*)ws, prefetch);
  int s = launch_status("attention_decode");
  if (s || ns == 1) return s;
  launch_pdl(combine_kernel<T, D>, dim3((unsigned)(B * H)), dim3(D), 0, st, (const float*)ws, ns, (T*)out, ld_out, (int)H);
  return launch_status("attention_decode_combine");
}

}  // namespace dec
}  // namespace gpt

extern "C" {

int64_t gpt_attention_decode_workspace_size(int64_t B, int64_t H, int64_t D, int64_t L) {
  if (B <= 0 || H <= 0 || D <= 0 || L <= 0) return 0;
  int sms = gpt::device_sm_count();
  if (sms <= 0) sms = 148;
  int ns = gpt::dec::num_splits(B, H, L, sms);
  if (ns == 1) return 0;
  return B * H * ns * (D + 2) * (int64_t)sizeof(float);
}

int gpt_attention_decode(const void* q, int64_t ld_q, const void* k_cache, const void* v_cache, void* out,
                         int64_t ld_out, int64_t B, int64_t H, int64_t D, int64_t Tmax, int64_t L,
                         const int64_t* len_dev, float scale, void* workspace, int dtype, void* stream) {
  GPT_CHECK_DTYPE(dtype);
  GPT_CHECK_SHAPE(B >= 0 && H > 0 && L >= (len_dev ? 0 : 1) && L <= Tmax && Tmax < (1LL << 30) && B * H < 65536 && ld_q >= H * D && ld_out >= H * D,
                  "gpt_attention_decode: bad sizes B=%lld H=%lld L=%lld Tmax=%lld", (long long)B, (long long)H,
                  (long long)L, (long long)Tmax);
  if (B == 0) return GPT_OK;
  GPT_CHECK_ARG(q && k_cache && v_cache && out, "gpt_attention_decode: null pointer");
  int64_t need = gpt_attention_decode_workspace_size(B, H, D, len_dev ? Tmax : L);
  GPT_CHECK_ARG(need == 0 || workspace, "gpt_attention_decode: workspace of %lld bytes required", (long long)need);
  size_t es = dtype == GPT_F32 ? 4 : 2;
  GPT_CHECK_ALIGN(gpt::aligned(q, 16) && gpt::aligned(k_cache, 16) && gpt::aligned(v_cache, 16) &&
                      (ld_q * es) % 16 == 0 && (D * es) % 16 == 0,
                  "gpt_attention_decode: needs 16-byte aligned q rows and cache rows");
  const float sl2 = scale * gpt::dec::kLog2e;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == GPT_BF16) {
    switch (D) {
      case 16: return gpt::dec::launch<__nv_bfloat16, 16>(q, ld_q, k_cache, v_cache, out, ld_out, B, H, Tmax, L, len_dev, sl2, workspace, st);
      case 32: return gpt::dec::launch<__nv_bfloat16, 32>(q, ld_q, k_cache, v_cache, out, ld_out, B, H, Tmax, L, len_dev, sl2, workspace, st);
      case 64: return gpt::dec::launch<__nv_bfloat16, 64>(q, ld_q, k_cache, v_cache, out, ld_out, B, H, Tmax, L, len_dev, sl2, workspace, st);
      case 128: return gpt::dec::launch<__nv_bfloat16, 128>(q, ld_q, k_cache, v_cache, out, ld_out, B, H, Tmax, L, len_dev, sl2, workspace, st);
      default: break;
    }
  } else {
    switch (D) {
      case 16: return gpt::dec::launch<float, 16>(q, ld_q, k_cache, v_cache, out, ld_out, B, H, Tmax, L, len_dev, sl2, workspace, st);
      case 32: return gpt::dec::launch<float, 32>(q, ld_q, k_cache, v_cache, out, ld_out, B, H, Tmax, L, len_dev, sl2, workspace, st);
      case 64: return gpt::dec::launch<float, 64>(q, ld_q, k_cache, v_cache, out, ld_out, B, H, Tmax, L, len_dev, sl2, workspace, st);
      case 128: return gpt::dec::launch<float, 128>(q, ld_q, k_cache, v_cache, out, ld_out, B, H, Tmax, L, len_dev, sl2, workspace, st);
      default: break;
    }
  }
  return gpt::fail(GPT_ERR_UNSUPPORTED, "gpt_attention_decode: head_dim %lld not in {16,32,64,128}", (long long)D);
}

}  // extern "C"
