// bf16 contraction for few activation rows (decode: M = sequences per GPU,
// 1..256): C[M, N] = epilogue(A[M, K] · W[N, K]ᵀ).
//
// With M that small the 128-row tile of gemm_tc_kernel leaves most SMs idle
// (N = 768 gives 3 CTAs) and the work is bound by streaming W from HBM.
// Here the operands swap roles: a CTA multiplies a 128-row slab of W (the
// MMA's M side) by all activation rows padded to Mp (the MMA's N side,
// 16..256) over a slice of K. The `splits` CTAs that share one slab form a
// thread-block cluster (split-K along the cluster): each leaves its fp32
// partial [Mp][128] in its own shared memory, one cluster barrier later
// every CTA reduces a slice of the rows by reading its peers' partials
// through distributed shared memory, applies bias / GELU / residual and
// stores C. No global workspace, no atomics, deterministic order.
//   warp 0 lane 0   TMA producer (W slab and A rows, 128B swizzle, ring)
//   warp 1          TMEM allocation (Mp columns); lane 0 issues tcgen05.mma
//   warps 0-3       epilogue: thread t owns slab row t (TMEM lane t).
#include "common.cuh"

namespace gpt {
namespace tc {

constexpr int kSkStages = 4;
constexpr int kSkThreads = 128;
constexpr int kSkMaxM = 256;
constexpr int kSkMaxSplits = 16;

struct SkParams {
  int M, N, K, Mp;
  int nkb, kb_per, splits;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* resid;
  __nv_bfloat16* C;
  int64_t ldr, ldc;
};

template <int EPI>
__device__ __forceinline__ void sk_store(const SkParams& p, int m, int n, float v) {
  if (EPI != GPT_EPI_NONE) v += __bfloat162float(p.bias[n]);
  if (EPI == GPT_EPI_BIAS_GELU) v = gelu_tanh<true>(v);
  if (EPI == GPT_EPI_BIAS_RESIDUAL) v += __bfloat162float(p.resid[(int64_t)m * p.ldr + n]);
  p.C[(int64_t)m * p.ldc + n] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Generic address of the same shared-memory location in cluster CTA `rank`;
// plain loads through it let the compiler keep many in flight.
__device__ __forceinline__ const float* peer_ptr(const float* local, uint32_t rank) {
  uint64_t out;
  asm("mapa.u64 %0, %1, %2;" : "=l"(out) : "l"(reinterpret_cast<uint64_t>(local)), "r"(rank));
  return reinterpret_cast<const float*>(out);
}

__host__ __device__ inline int sk_ring_bytes(int Mp) { return kSkStages * (128 * BK * 2 + Mp * BK * 2); }
__host__ __device__ inline int sk_smem_bytes(int Mp) { return 1024 + sk_ring_bytes(Mp) + (2 * kSkStages + 1) * 8 + 16; }

template <int EPI>
__global__ void __launch_bounds__(kSkThreads)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA,
                       const SkParams p) {
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smem_dyn + 1023) & ~(uintptr_t)1023);
  constexpr int kWBytes = 128 * BK * 2;
  const int aBytes = p.Mp * BK * 2;
  uint8_t* ringW = base;
  uint8_t* ringA = base + kSkStages * kWBytes;
  // After the main loop the ring is idle and holds this CTA's fp32 partial
  // [Mp][128] (Mp*512 bytes <= ring size for every Mp).
  float* part = reinterpret_cast<float*>(base);
  uint64_t* bars = (uint64_t*)(base + sk_ring_bytes(p.Mp));
  uint64_t* full = bars;
  uint64_t* empty = bars + kSkStages;
  uint64_t* done = bars + 2 * kSkStages;
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * kSkStages + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int split = p.splits > 1 ? (int)cluster_ctarank() : 0;
  const int n0 = tile * 128;
  const int kb0 = split * p.kb_per;
  const int kb1 = min(p.nkb, kb0 + p.kb_per);
  const uint32_t tcols = p.Mp <= 32 ? 32u : p.Mp <= 64 ? 64u : p.Mp <= 128 ? 128u : 256u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSkStages; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), 1);
    }
    mbar_init(smem_addr(done), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(tcols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    const uint32_t bytes = (uint32_t)(kWBytes + aBytes);
    // Weights do not depend on earlier kernels: the first ring slots are
    // filled with W before waiting for the previous kernel (programmatic
    // dependent launch), the activation rows after.
    const int pre = min(kb1 - kb0, kSkStages);
    for (int i = 0; i < pre; ++i) {
      const uint32_t fb = smem_addr(&full[i]);
      mbar_expect_tx(fb, bytes);
      tma_load_2d(smem_addr(ringW + i * kWBytes), &tmW, fb, (kb0 + i) * BK, n0);
    }
    pdl_wait();
    pdl_trigger();
    for (int i = 0; i < pre; ++i)
      tma_load_2d(smem_addr(ringA + i * aBytes), &tmA, smem_addr(&full[i]), (kb0 + i) * BK, 0);
    int stage = pre % kSkStages;
    uint32_t phase = pre == kSkStages ? 1u : 0u;
    for (int kb = kb0 + pre; kb < kb1; ++kb) {
      if (!mbar_wait(smem_addr(&empty[stage]), phase ^ 1)) break;
      const uint32_t fb = smem_addr(&full[stage]);
      mbar_expect_tx(fb, bytes);
      tma_load_2d(smem_addr(ringW + stage * kWBytes), &tmW, fb, kb * BK, n0);
      tma_load_2d(smem_addr(ringA + stage * aBytes), &tmA, fb, kb * BK, 0);
      if (++stage == kSkStages) { stage = 0; phase ^= 1; }
    }
  } else if (warp == 1 && lane == 0) {
    // kind::f16, D fp32, A = W slab (128 rows), B = activation rows (Mp), both K-major.
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.Mp >> 3) << 17) |
                           ((uint32_t)(128 >> 4) << 24);
    int stage = 0;
    uint32_t phase = 0;
    for (int kb = kb0; kb < kb1; ++kb) {
      if (!mbar_wait(smem_addr(&full[stage]), phase)) break;
      tc_fence_after();
      const uint64_t wd = desc_sw128(smem_addr(ringW + stage * kWBytes));
      const uint64_t ad = desc_sw128(smem_addr(ringA + stage * aBytes));
#pragma unroll
      for (int k = 0; k < BK / 16; ++k)
        tc_mma(tmem, wd + (uint64_t)(2 * k), ad + (uint64_t)(2 * k), idesc, (kb > kb0 || k > 0) ? 1u : 0u);
      tc_commit(smem_addr(&empty[stage]));
      if (++stage == kSkStages) { stage = 0; phase ^= 1; }
    }
    tc_commit(smem_addr(done));  // also covers an empty K slice (no MMA issued)
  }
  __syncwarp();
  if (!(warp == 0 && lane == 0)) pdl_wait();
  const bool ok = mbar_wait(smem_addr(done), 0);
  tc_fence_after();

  const int nl = warp * 32 + lane;  // row of the W slab == TMEM lane
  const int n = n0 + nl;
  const bool n_ok = n < p.N;
  const bool has_k = kb1 > kb0;
  const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
  if (p.splits == 1) {
    for (int c = 0; c < p.Mp && ok; c += 32) {
      uint32_t r[32];
      tmem_ld32(lane_base + (uint32_t)c, r);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int m = c + j;
        if (m < p.M && n_ok) sk_store<EPI>(p, m, n, __uint_as_float(r[j]));
      }
    }
  } else {
    // own partial -> shared memory (the ring is no longer read by TMA or MMA)
    for (int c = 0; c < p.Mp; c += 32) {
      uint32_t r[32];
      if (ok && has_k) tmem_ld32(lane_base + (uint32_t)c, r);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c + j < p.Mp) part[(c + j) * 128 + nl] = (ok && has_k) ? __uint_as_float(r[j]) : 0.f;
    }
    cluster_sync();  // every partial of the cluster is visible
    const int mchunk = (p.M + p.splits - 1) / p.splits;
    const int m_lo = split * mchunk, m_hi = min(p.M, m_lo + mchunk);
    float bn = 0.f;
    if (EPI != GPT_EPI_NONE && n_ok) bn = __bfloat162float(p.bias[n]);
    for (int m0 = m_lo; m0 < m_hi; m0 += 8) {
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int s = 0; s < p.splits; ++s) {
        const float* src = peer_ptr(part, (uint32_t)s) + m0 * 128 + nl;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (m0 + j < m_hi) v[j] += src[j * 128];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int m = m0 + j;
        if (m < m_hi && n_ok) {
          float x = v[j] + bn;
          if (EPI == GPT_EPI_BIAS_GELU) x = gelu_tanh<true>(x);
          if (EPI == GPT_EPI_BIAS_RESIDUAL) x += __bfloat162float(p.resid[(int64_t)m * p.ldr + n]);
          p.C[(int64_t)m * p.ldc + n] = __float2bfloat16_rn(x);
        }
      }
    }
    cluster_sync();  // peers have finished reading this CTA's shared memory
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols));
  }
}

struct SkPlan {
  int Mp, tiles, nkb, kb_per, splits;
};

// Splits: enough CTAs for about two per SM, at most the cluster size limit,
// never an empty K slice.
inline SkPlan sk_plan(int64_t M, int64_t N, int64_t K, int sms, int max_splits) {
  SkPlan pl;
  pl.Mp = (int)(((M + 15) / 16) * 16);
  pl.tiles = (int)((N + 127) / 128);
  pl.nkb = (int)((K + BK - 1) / BK);
  int want = (2 * sms + pl.tiles - 1) / pl.tiles;
  static const int forced = [] {
    const char* e = getenv("GPT_SKINNY_SPLITS");
    return e ? atoi(e) : 0;
  }();
  if (forced > 0) want = forced;
  if (want > max_splits) want = max_splits;
  if (want > pl.nkb) want = pl.nkb;
  if (want < 1) want = 1;
  pl.kb_per = (pl.nkb + want - 1) / want;
  pl.splits = (pl.nkb + pl.kb_per - 1) / pl.kb_per;
  return pl;
}

template <int EPI>
static int sk_launch(const CUtensorMap& tw, const CUtensorMap& ta, const SkParams& p, int tiles, int smem,
                     cudaStream_t st) {
  auto kern = gemm_skinny_kernel<EPI>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)tiles, (unsigned)p.splits, 1);
  cfg.blockDim = dim3(kSkThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)p.splits;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, ta, p);
  if (e != cudaSuccess) return fail(GPT_ERR_CUDA, "gemm_skinny launch: %s", cudaGetErrorString(e));
  return launch_status("gemm_skinny");
}

// Largest cluster this kernel may use on the current device (8 portable,
// 16 where the non-portable attribute is accepted); set up once per device.
template <int EPI>
static int sk_setup(int* max_splits) {
  static int cached[64] = {0};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(GPT_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> g(mu);
  if (cached[dev] == 0) {
    auto kern = gemm_skinny_kernel<EPI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sk_smem_bytes(kSkMaxM));
    if (e != cudaSuccess) return fail(GPT_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    // Clusters above 8 CTAs are non-portable; they are used only when the
    // attribute is accepted and a 16-CTA cluster of the largest footprint fits.
    int ms = 8;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, kSkMaxSplits, 1);
      cfg.blockDim = dim3(kSkThreads, 1, 1);
      cfg.dynamicSmemBytes = (size_t)sk_smem_bytes(kSkMaxM);
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1;
      attr[0].val.clusterDim.y = kSkMaxSplits;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) == cudaSuccess && clusters > 0) ms = kSkMaxSplits;
    }
    cudaGetLastError();
    cached[dev] = ms;
  }
  *max_splits = cached[dev];
  return GPT_OK;
}

template <int EPI>
static int gemm_skinny_epi(const void* A, int64_t lda, const void* W, const SkParams& p0, int64_t M, int64_t N,
                           int64_t K, cudaStream_t st) {
  int max_splits = 8;
  int s = sk_setup<EPI>(&max_splits);
  if (s) return s;
  int sms = device_sm_count();
  if (sms <= 0) return fail(GPT_ERR_CUDA, "no CUDA device");
  SkPlan pl = sk_plan(M, N, K, sms, max_splits);
  CUtensorMap tw, ta;
  s = make_map(&tw, W, N, K, K, 128);
  if (s) return s;
  s = make_map(&ta, A, M, K, lda, pl.Mp);
  if (s) return s;
  SkParams p = p0;
  p.Mp = pl.Mp;
  p.nkb = pl.nkb;
  p.kb_per = pl.kb_per;
  p.splits = pl.splits;
  return sk_launch<EPI>(tw, ta, p, pl.tiles, sk_smem_bytes(pl.Mp), st);
}

// Serves bf16 requests with M <= kSkMaxM rows.
int gemm_skinny(const void* A, int64_t lda, const void* W, const void* bias, const void* R, int64_t ldr, void* C,
                int64_t ldc, int64_t M, int64_t N, int64_t K, int epi, cudaStream_t st) {
  SkParams p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.bias = (const __nv_bfloat16*)bias;
  p.resid = (const __nv_bfloat16*)R;
  p.C = (__nv_bfloat16*)C;
  p.ldr = ldr;
  p.ldc = ldc;
  switch (epi) {
    case GPT_EPI_NONE: return gemm_skinny_epi<GPT_EPI_NONE>(A, lda, W, p, M, N, K, st);
    case GPT_EPI_BIAS: return gemm_skinny_epi<GPT_EPI_BIAS>(A, lda, W, p, M, N, K, st);
    case GPT_EPI_BIAS_GELU: return gemm_skinny_epi<GPT_EPI_BIAS_GELU>(A, lda, W, p, M, N, K, st);
    default: return gemm_skinny_epi<GPT_EPI_BIAS_RESIDUAL>(A, lda, W, p, M, N, K, st);
  }
}

}  // namespace tc
}  // namespace gpt
