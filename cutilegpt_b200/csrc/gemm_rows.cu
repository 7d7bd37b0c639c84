// bf16 contraction for the decode step's few activation rows (M <= 128
// sequences per GPU): C[M, N] = epilogue(A[M, K] · W[N, K]ᵀ), with the
// decode-step extras (LayerNorm folded in, row sums of the output for the
// next fold, K/V append) — the few-row counterpart of the reference's
// cutile_linear_bias (cutile_gpt/kernels/linear.py:164-222), which the
// reference only ever runs on whole prompts.
//
// Layout of the work: the activation rows are the MMA's M side (M = 128,
// rows past M are never loaded and their TMEM lanes never read), a CTA owns
// a tile of BN = 64 (32, 16 when N needs it) weight rows (the MMA's N side)
// and a slice of K; the S CTAs of a thread-block cluster share one tile and
// split its K. Every CTA reads the activation rows of its K slice from L2,
// and the L2 traffic of all CTAs together is what bounds the kernel: it is
// (N / BN) x M x K x 2 bytes, so wide tiles with split-K beat 16-wide tiles
// that each read all of K. So:
//   * the CTA's whole weight slice (BN x K_slice bf16, <= 48 KB) is
//     requested by TMA before the programmatic-dependent-launch wait:
//     weights stream from HBM while the previous kernel is still running;
//   * after the wait only the activation rows move (L2 -> shared memory,
//     4-stage ring), the MMAs follow them k-block by k-block;
//   * the BN-column partial of the S CTAs is reduce-scattered over
//     distributed shared memory in units of (row, 16 columns): unit u goes
//     to cluster rank u % S, every CTA sends its partial of a unit with four
//     `st.async` remote stores counted on the owner's mbarrier, and the owner
//     adds the S partials in rank order (deterministic);
//   * the epilogue is one thread per owned unit: LayerNorm fold (mean / rstd
//     from exact fp64 row sums), bias, tanh-GELU, residual, bf16 store of 32
//     contiguous bytes, K/V append of those bytes, and the (sum, sum of
//     squares) of the stored row segment added in fp64 to the output row
//     sums. Those are sums of bf16 values and their squares, exact in fp64
//     for any realistic range of magnitudes, so the atomically accumulated
//     totals do not depend on the order of arrival.
// Threads: warp 0 lane 0 TMA producer, warp 1 TMEM allocation and lane 0
// MMA issue, then all 128 threads read the accumulator (thread = TMEM lane
// = row) and run the epilogue. Every wait is bounded.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace gpt {
namespace rows {

using tc::BK;
using tc::desc_sw128;
using tc::mbar_expect_tx;
using tc::mbar_init;
using tc::mbar_wait;
using tc::smem_addr;
using tc::tc_commit;
using tc::tc_fence_after;
using tc::tc_fence_before;
using tc::tc_mma;
using tc::tma_load_2d;

constexpr int kThreads = 128;
constexpr int kStages = 4;
constexpr int kMaxM = 128;
constexpr int kMaxSplits = 8;                 // cluster size (portable maximum)
constexpr int kMaxWBytes = 48 * 1024;         // weight slice per CTA
constexpr int kMaxSmem = 227 * 1024;

struct RowsParams {
  int M, N, K, Mp;
  int nkb, kb_per, splits, stages;
  int own_max;             // units (row, 16 columns) owned by one cluster rank, rounded up
  const __nv_bfloat16* bias;
  const __nv_bfloat16* resid;
  __nv_bfloat16* C;
  int64_t ldr, ldc;
  int vec_c, vec_r;        // 16-byte aligned C / residual row segments
  const double* ln_sums;   // [M][2] (sum, sum of squares) of A's rows: LayerNorm folded in
  const float* ln_u;       // [N] row sums of the gamma-scaled weight
  const float* ln_v;       // [N] W . beta + bias (replaces bias)
  float ln_eps;
  double ln_inv_k;
  double* sums_out;        // [M][2] += (sum, sum of squares) of C's stored rows
  __nv_bfloat16* kc;       // K/V append of a QKV output: caches [M][H][Tmax][D]
  __nv_bfloat16* vc;
  int kv_C, kv_D, kv_H;
  int64_t kv_tmax, kv_pos0;
  const int64_t* kv_pos;
};

// Activation stage: the Mp loaded rows x 64 k (Mp * 128 bytes, whole SW128
// atoms of 8 rows). The MMA reads 128 rows from a stage's base; rows past Mp
// fall into the next stage or the guard after the last one, and their TMEM
// lanes are never read.
__host__ __device__ inline int rows_smem_bytes(int bn, int stages, int kb_per, int splits, int own_max, int Mp) {
  return 1024 + stages * Mp * BK * 2 + (128 - Mp) * BK * 2 + kb_per * bn * BK * 2 +
         (splits > 1 ? splits * own_max * 64 : 0) + 16 * 8;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t local, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(local), "r"(rank));
  return out;
}
__device__ __forceinline__ void st_async_v4(uint32_t remote, const float* v, uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(remote),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "r"(remote_bar)
      : "memory");
}
// 32 lanes x 16 consecutive fp32 columns: thread t of the warp gets TMEM lane (quadrant * 32 + t).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}

// Inputs of one epilogue unit (row m, columns n0 .. n0 + 15) that earlier
// kernels do not write (weights) or that are final before this kernel runs
// (residual row, row sums): loaded while the MMAs run where possible.
template <int EPI>
struct UnitIn {
  float cb[16], cu[16], rres[16];
  float mean, rstd;
};

template <int EPI>
__device__ __forceinline__ void load_unit(const RowsParams& p, int m, int n0, UnitIn<EPI>& in) {
  const bool ln = p.ln_sums != nullptr;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    in.cu[j] = 0.f;
    in.rres[j] = 0.f;
    if (ln) {
      in.cu[j] = p.ln_u[n0 + j];
      in.cb[j] = p.ln_v[n0 + j];
    } else {
      in.cb[j] = EPI != GPT_EPI_NONE ? __bfloat162float(p.bias[n0 + j]) : 0.f;
    }
  }
  in.mean = 0.f;
  in.rstd = 1.f;
  if (EPI == GPT_EPI_BIAS_RESIDUAL) {
    const __nv_bfloat16* rp = p.resid + (int64_t)m * p.ldr + n0;
    if (p.vec_r) {
      const uint4 a = *reinterpret_cast<const uint4*>(rp);
      const uint4 b = *reinterpret_cast<const uint4*>(rp + 8);
      const __nv_bfloat16* e0 = reinterpret_cast<const __nv_bfloat16*>(&a);
      const __nv_bfloat16* e1 = reinterpret_cast<const __nv_bfloat16*>(&b);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        in.rres[j] = __bfloat162float(e0[j]);
        in.rres[8 + j] = __bfloat162float(e1[j]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) in.rres[j] = __bfloat162float(rp[j]);
    }
  }
  if (ln) {
    const double2 s = *reinterpret_cast<const double2*>(p.ln_sums + 2 * (int64_t)m);
    const double mu = s.x * p.ln_inv_k;
    const double var = fmax(s.y * p.ln_inv_k - mu * mu, 0.0);
    in.mean = (float)mu;
    in.rstd = rsqrtf((float)var + p.ln_eps);
  }
}

template <int EPI>
__device__ __forceinline__ void store_unit(const RowsParams& p, int m, int n0, const float* acc,
                                           const UnitIn<EPI>& in) {
  const bool ln = p.ln_sums != nullptr;
  __align__(16) __nv_bfloat16 y[16];
  double s1 = 0.0, s2 = 0.0;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    float x = ln ? in.rstd * (acc[j] - in.mean * in.cu[j]) + in.cb[j] : acc[j] + in.cb[j];
    if (EPI == GPT_EPI_BIAS_GELU) x = gelu_tanh<true>(x);
    if (EPI == GPT_EPI_BIAS_RESIDUAL) x += in.rres[j];
    y[j] = __float2bfloat16_rn(x);
    const double yd = (double)__bfloat162float(y[j]);
    s1 += yd;
    s2 = fma(yd, yd, s2);
  }
  __nv_bfloat16* dst = p.C + (int64_t)m * p.ldc + n0;
  if (p.vec_c) {
    reinterpret_cast<uint4*>(dst)[0] = reinterpret_cast<const uint4*>(y)[0];
    reinterpret_cast<uint4*>(dst)[1] = reinterpret_cast<const uint4*>(y)[1];
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) dst[j] = y[j];
  }
  if (p.kc && n0 >= p.kv_C) {
    // k or v part of a QKV row; 16 | head_dim keeps the unit inside one head
    const int idx = n0 - p.kv_C;
    const int which = idx / p.kv_C, hd = idx - which * p.kv_C;
    const int h = hd / p.kv_D, d = hd - h * p.kv_D;
    const int64_t pos = p.kv_pos0 + (p.kv_pos ? *p.kv_pos : 0);
    if (pos < p.kv_tmax) {
      __nv_bfloat16* kd = (which == 0 ? p.kc : p.vc) + (((int64_t)m * p.kv_H + h) * p.kv_tmax + pos) * p.kv_D + d;
      reinterpret_cast<uint4*>(kd)[0] = reinterpret_cast<const uint4*>(y)[0];
      reinterpret_cast<uint4*>(kd)[1] = reinterpret_cast<const uint4*>(y)[1];
    } else if (m == 0) {
      record_device_error(GPT_DEVERR_INDEX);
    }
  }
  if (p.sums_out) {
    atomicAdd(p.sums_out + 2 * (int64_t)m, s1);
    atomicAdd(p.sums_out + 2 * (int64_t)m + 1, s2);
  }
}

template <int EPI, int BN>
__global__ void __launch_bounds__(kThreads, 2)
    gemm_rows_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                     const RowsParams p) {
  constexpr int NC = BN / 16;                // 16-column units per row of the tile
  constexpr int kWBytes = BN * BK * 2;       // one weight k-block
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smem_dyn + 1023) & ~(uintptr_t)1023);
  const int a_stage = p.Mp * BK * 2;
  uint8_t* ringA = base;
  uint8_t* wbuf = base + p.stages * a_stage + (128 - p.Mp) * BK * 2;
  float* recv = reinterpret_cast<float*>(wbuf + p.kb_per * kWBytes);   // [S][own_max][16]
  uint64_t* bars = reinterpret_cast<uint64_t*>(recv + (p.splits > 1 ? p.splits * p.own_max * 16 : 0));
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* wfull = bars + 2 * kStages;
  uint64_t* done = bars + 2 * kStages + 1;
  uint64_t* recv_full = bars + 2 * kStages + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 3);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x;
  const int S = p.splits;
  const bool clustered = S > 1;
  const int split = clustered ? (int)cluster_rank() : 0;
  const int n_tile = tile * BN;
  const int kb0 = split * p.kb_per;
  const int kb1 = min(p.nkb, kb0 + p.kb_per);
  const int nk = kb1 - kb0;  // >= 1 (the host never makes an empty slice)
  const int units = p.M * NC;                                      // (row, 16 columns) units of real rows
  const int owned = units > split ? (units - 1 - split) / S + 1 : 0;   // units this rank finishes

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), 1);
    }
    mbar_init(smem_addr(wfull), 1);
    mbar_init(smem_addr(done), 1);
    mbar_init(smem_addr(recv_full), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (clustered) mbar_expect_tx(smem_addr(recv_full), (uint32_t)(owned * (S - 1) * 64));
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(BN < 32 ? 32 : BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  // Every receive barrier of the cluster is initialised before any peer can send.
  if (clustered) {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  }
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    // The weight slice does not depend on earlier kernels: all of it is in
    // flight before the dependency wait.
    mbar_expect_tx(smem_addr(wfull), (uint32_t)(nk * kWBytes));
    for (int i = 0; i < nk; ++i)
      tma_load_2d(smem_addr(wbuf + i * kWBytes), &tmW, smem_addr(wfull), (kb0 + i) * BK, n_tile);
    pdl_wait();
    pdl_trigger();
    const uint32_t abytes = (uint32_t)(p.Mp * BK * 2);
    for (int i = 0; i < nk; ++i) {
      const int s = i % p.stages, r = i / p.stages;
      if (r > 0 && !mbar_wait(smem_addr(&empty[s]), (uint32_t)((r - 1) & 1))) break;
      mbar_expect_tx(smem_addr(&full[s]), abytes);
      tma_load_2d(smem_addr(ringA + s * a_stage), &tmA, smem_addr(&full[s]), (kb0 + i) * BK, 0);
    }
  } else if (warp == 1 && lane == 0) {
    // kind::f16, D fp32, A = activation rows (M = 128), B = weight rows (N = BN), both K-major.
    constexpr uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                               ((uint32_t)(128 >> 4) << 24);
    bool ok = mbar_wait(smem_addr(wfull), 0);
    for (int i = 0; i < nk && ok; ++i) {
      const int s = i % p.stages, r = i / p.stages;
      if (!mbar_wait(smem_addr(&full[s]), (uint32_t)(r & 1))) break;
      tc_fence_after();
      const uint64_t ad = desc_sw128(smem_addr(ringA + s * a_stage));
      const uint64_t wd = desc_sw128(smem_addr(wbuf + i * kWBytes));
#pragma unroll
      for (int k = 0; k < BK / 16; ++k)
        tc_mma(tmem, ad + (uint64_t)(2 * k), wd + (uint64_t)(2 * k), idesc, (i > 0 || k > 0) ? 1u : 0u);
      tc_commit(smem_addr(&empty[s]));
    }
    tc_commit(smem_addr(done));
  }
  __syncwarp();
  if (tid != 0) pdl_wait();

  // Inputs of this thread's first epilogue unit, fetched while the MMAs run.
  UnitIn<EPI> in;
  const int u_first = clustered ? tid * S + split : tid * NC;   // unit index (row-major: u = m * NC + c)
  if (u_first < units) load_unit<EPI>(p, u_first / NC, n_tile + (u_first % NC) * 16, in);

  const bool ok = mbar_wait(smem_addr(done), 0);
  tc_fence_after();
  const int m = tid;   // TMEM lane of this thread = accumulator row
  const bool row_ok = m < p.M;
  if (!clustered) {
    // One rank: the thread finishes the NC units of its row directly.
#pragma unroll 1
    for (int c = 0; c < NC; ++c) {
      float acc[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 16), acc);   // whole warps
      if (row_ok && ok) {
        if (c > 0) load_unit<EPI>(p, m, n_tile + c * 16, in);
        store_unit<EPI>(p, m, n_tile + c * 16, acc, in);
      }
    }
  } else {
    // Reduce-scatter: the partial of unit u goes to slot [split][u / S] of rank u % S.
    const uint32_t recv_s = smem_addr(recv);
    const uint32_t bar_s = smem_addr(recv_full);
#pragma unroll 1
    for (int c = 0; c < NC; ++c) {
      float acc[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 16), acc);
      if (!row_ok) continue;
      if (!ok) {
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = 0.f;
      }
      const int u = m * NC + c;
      const int owner = u % S, li = u / S;
      const uint32_t off = (uint32_t)(((split * p.own_max) + li) * 64);
      if (owner == split) {
        float4* d = reinterpret_cast<float4*>(recv + (split * p.own_max + li) * 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) d[q] = make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
      } else {
        const uint32_t dst = map_to_rank(recv_s + off, (uint32_t)owner);
        const uint32_t bar = map_to_rank(bar_s, (uint32_t)owner);
#pragma unroll
        for (int q = 0; q < 4; ++q) st_async_v4(dst + q * 16, acc + 4 * q, bar);
      }
    }
    __syncthreads();   // this rank's own partials are in shared memory
    const bool got = owned > 0 ? mbar_wait(smem_addr(recv_full), 0) : true;
#pragma unroll 1
    for (int li = tid; li < owned; li += kThreads) {
      const int u = li * S + split;
      const int um = u / NC, n0 = n_tile + (u % NC) * 16;
      if (li != tid) load_unit<EPI>(p, um, n0, in);
      float acc[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[j] = 0.f;
      for (int s = 0; s < S; ++s) {   // fixed order: rank 0, 1, ...
        const float4* src = reinterpret_cast<const float4*>(recv + (s * p.own_max + li) * 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v = src[q];
          acc[4 * q] += v.x;
          acc[4 * q + 1] += v.y;
          acc[4 * q + 2] += v.z;
          acc[4 * q + 3] += v.w;
        }
      }
      if (ok && got) store_unit<EPI>(p, um, n0, acc, in);
    }
  }
  // No closing cluster barrier: every write into this CTA's shared memory is
  // a partial counted on its receive barrier, which it has waited for, so no
  // peer can still be writing here when it leaves.
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN < 32 ? 32 : BN));
  }
}

// Row sums for the first LayerNorm fold of a decode step: sums[m] = (sum,
// sum of squares) over the C values of row m of x (fp64), and zero[0, n)
// cleared for the row-sum accumulations of the step's later GEMMs.
template <typename T>
__global__ void __launch_bounds__(256) row_sums_kernel(const T* __restrict__ x, int64_t ld, int M, int C,
                                                       double* __restrict__ sums, double* __restrict__ zero,
                                                       int64_t n_zero) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = blockIdx.x * 8 + warp;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_zero; i += (int64_t)gridDim.x * blockDim.x)
    zero[i] = 0.0;
  if (m >= M) return;
  double s1 = 0.0, s2 = 0.0;
  for (int c = lane; c < C; c += 32) {
    const double v = (double)Tr<T>::to_f(x[(int64_t)m * ld + c]);
    s1 += v;
    s2 = fma(v, v, s2);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  }
  if (lane == 0) {
    sums[2 * (int64_t)m] = s1;
    sums[2 * (int64_t)m + 1] = s2;
  }
}

template <int EPI, int BN>
static int rows_launch(const CUtensorMap& ta, const CUtensorMap& tw, const RowsParams& p, int tiles, int smem,
                       cudaStream_t st) {
  auto kern = gemm_rows_kernel<EPI, BN>;
  static bool attr_done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(GPT_ERR_UNSUPPORTED, "device %d", dev);
  {
    std::lock_guard<std::mutex> g(mu);
    if (!attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
      if (e != cudaSuccess) return fail(GPT_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      attr_done[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)tiles, (unsigned)p.splits, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = (unsigned)p.splits;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tw, p);
  if (e != cudaSuccess) return fail(GPT_ERR_CUDA, "gemm_rows launch: %s", cudaGetErrorString(e));
  return launch_status("gemm_rows");
}

template <int BN>
static int rows_dispatch(int epi, const CUtensorMap& ta, const CUtensorMap& tw, const RowsParams& p, int tiles,
                         int smem, cudaStream_t st) {
  switch (epi) {
    case GPT_EPI_NONE: return rows_launch<GPT_EPI_NONE, BN>(ta, tw, p, tiles, smem, st);
    case GPT_EPI_BIAS: return rows_launch<GPT_EPI_BIAS, BN>(ta, tw, p, tiles, smem, st);
    case GPT_EPI_BIAS_GELU: return rows_launch<GPT_EPI_BIAS_GELU, BN>(ta, tw, p, tiles, smem, st);
    default: return rows_launch<GPT_EPI_BIAS_RESIDUAL, BN>(ta, tw, p, tiles, smem, st);
  }
}

// Tile width and split-K of one decode GEMM. The widest tile that divides N
// (it sets the L2 traffic of the activation rows, (N / BN) x Mp x K x 2
// bytes); then the split count that brings tiles x splits closest to one CTA
// per SM, within the cluster size and a 48 KB weight slice per CTA.
struct RowsConfig {
  int bn, splits, kb_per;
};
static bool choose_config(int64_t N, int nkb, int sms, RowsConfig* out) {
  for (int bn : {64, 32, 16}) {
    if (N % bn) continue;
    const int tiles = (int)(N / bn);
    const int kb_cap = kMaxWBytes / (bn * BK * 2);
    const int need = (nkb + kb_cap - 1) / kb_cap;   // splits the weight-slice cap requires
    if (need > kMaxSplits) continue;                // K too long for this width
    const int fill = std::min(std::max(1, (sms + tiles / 2) / tiles), kMaxSplits);
    const int want = std::min(std::max(fill, need), nkb);
    const int kb_per = (nkb + want - 1) / want;
    *out = {bn, (nkb + kb_per - 1) / kb_per, kb_per};
    return true;
  }
  return false;
}

}  // namespace rows

namespace tc {
// Shapes the few-row kernel serves: up to 128 rows, N a multiple of 16,
// 16-byte aligned operands and row pitches (TMA), K slices of whole 64-wide
// k-blocks (a ragged K tail is zero-filled by TMA on both operands).
bool rows_eligible(const void* A, int64_t lda, const void* W, const void* C, int64_t ldc, int64_t M, int64_t N,
                   int64_t K) {
  return M >= 1 && M <= rows::kMaxM && N % 16 == 0 && N / 16 < 65536 && K >= 1 && K % 8 == 0 &&
         K <= 16384 && lda % 8 == 0 && aligned(A, 16) && aligned(W, 16) && C != nullptr && ldc >= N;
}

int gemm_rows(const void* A, int64_t lda, const void* W, const void* bias, const void* R, int64_t ldr, void* C,
              int64_t ldc, int64_t M, int64_t N, int64_t K, int epi, const gpt_gemm_fusion* f, cudaStream_t st) {
  using namespace rows;
  const int sms = device_sm_count();
  if (sms <= 0) return fail(GPT_ERR_CUDA, "no CUDA device");
  RowsParams p = {};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.Mp = (int)((M + 7) / 8 * 8);
  p.nkb = (int)((K + BK - 1) / BK);
  RowsConfig rc;
  if (!choose_config(N, p.nkb, sms, &rc))
    return fail(GPT_ERR_UNSUPPORTED, "gemm_rows: K = %lld too large for N = %lld", (long long)K, (long long)N);
  const int tiles = (int)(N / rc.bn);
  p.kb_per = rc.kb_per;
  p.splits = rc.splits;
  p.own_max = (p.Mp * (rc.bn / 16) + p.splits - 1) / p.splits;
  p.stages = std::min(kStages, p.kb_per);
  p.bias = (const __nv_bfloat16*)bias;
  p.resid = (const __nv_bfloat16*)R;
  p.C = (__nv_bfloat16*)C;
  p.ldr = ldr;
  p.ldc = ldc;
  p.vec_c = aligned(C, 16) && ldc % 8 == 0;
  p.vec_r = R && aligned(R, 16) && ldr % 8 == 0;
  if (f) {
    p.ln_sums = f->ln_sums;
    p.ln_u = f->ln_u;
    p.ln_v = f->ln_v;
    p.ln_eps = f->ln_eps;
    p.sums_out = f->row_sums;
    p.kc = (__nv_bfloat16*)f->k_cache;
    p.vc = (__nv_bfloat16*)f->v_cache;
    p.kv_C = (int)(f->kv_heads * f->kv_dim);
    p.kv_D = (int)f->kv_dim;
    p.kv_H = (int)f->kv_heads;
    p.kv_tmax = f->kv_tmax;
    p.kv_pos0 = f->kv_pos0;
    p.kv_pos = f->kv_pos_dev;
    if (p.kc && (f->kv_dim % 16 != 0 || !aligned(f->k_cache, 16) || !aligned(f->v_cache, 16)))
      return fail(GPT_ERR_ALIGN, "gemm_rows: the K/V append needs 16-byte aligned caches and head_dim %% 16 == 0");
  }
  p.ln_inv_k = 1.0 / (double)K;
  CUtensorMap ta, tw;
  int s = make_map(&ta, A, M, K, lda, p.Mp);
  if (s) return s;
  s = make_map(&tw, W, N, K, K, rc.bn);
  if (s) return s;
  const int smem = rows_smem_bytes(rc.bn, p.stages, p.kb_per, p.splits, p.own_max, p.Mp);
  if (smem > kMaxSmem) return fail(GPT_ERR_UNSUPPORTED, "gemm_rows: shared memory %d bytes", smem);
  switch (rc.bn) {
    case 64: return rows_dispatch<64>(epi, ta, tw, p, tiles, smem, st);
    case 32: return rows_dispatch<32>(epi, ta, tw, p, tiles, smem, st);
    default: return rows_dispatch<16>(epi, ta, tw, p, tiles, smem, st);
  }
}
}  // namespace tc
}  // namespace gpt

extern "C" int gpt_row_sums(const void* x, int64_t ld, int64_t M, int64_t C, double* sums, double* zero,
                            int64_t n_zero, int dtype, void* stream) {
  GPT_CHECK_DTYPE(dtype);
  GPT_CHECK_SHAPE(M >= 0 && C > 0 && ld >= C && n_zero >= 0 && M < (1LL << 31),
                  "gpt_row_sums: bad sizes M=%lld C=%lld ld=%lld", (long long)M, (long long)C, (long long)ld);
  if (M == 0 && n_zero == 0) return GPT_OK;
  GPT_CHECK_ARG(x && sums && (n_zero == 0 || zero), "gpt_row_sums: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int blocks = (int)std::max<int64_t>((M + 7) / 8, std::min<int64_t>((n_zero + 255) / 256, 148));
  if (dtype == GPT_BF16)
    gpt::launch_pdl(gpt::rows::row_sums_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st,
                    (const __nv_bfloat16*)x, ld, (int)M, (int)C, sums, zero, n_zero);
  else
    gpt::launch_pdl(gpt::rows::row_sums_kernel<float>, dim3(blocks), dim3(256), 0, st, (const float*)x, ld, (int)M,
                    (int)C, sums, zero, n_zero);
  return gpt::launch_status("row_sums");
}
