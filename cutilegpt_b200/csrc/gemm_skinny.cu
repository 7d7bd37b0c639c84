// bf16 contraction for few activation rows (decode: M = sequences per GPU,
// 1..256): C[M, N] = epilogue(A[M, K] · W[N, K]ᵀ).
//
// With M that small the 128-row tile of gemm_tc_kernel leaves most SMs idle
// (N = 768 gives 3 CTAs) and the work is bound by streaming W from HBM.
// Here the operands swap roles: a CTA multiplies a 128-row slab of W (the
// MMA's M side) by all activation rows padded to Mp (the MMA's N side,
// 16..256) over a slice of K. The `splits` CTAs that share one slab form a
// thread-block cluster (split-K along the cluster). After its MMAs each CTA
// stages its fp32 partial [Mp][128] in shared memory and pushes the row
// block owned by every cluster CTA into that CTA's receive buffer with one
// `cp.async.bulk` shared::cta -> shared::cluster copy, counted on the
// owner's mbarrier. Each owner then sums its rows over the peers in a fixed
// order (deterministic, no global workspace, no atomics), applies bias /
// GELU / residual (and, in the fused variant, the LayerNorm fold, output row
// statistics and the KV append) and stores C with 8-byte stores.
//   warp 0 lane 0   TMA producer (W slab and A rows, 128B swizzle, ring)
//   warp 1          TMEM allocation (Mp columns); lane 0 issues tcgen05.mma
//   warps 0-3       epilogue: TMEM lane t = slab row t, then one thread per
//                   (owner row, 4 output columns) for the reduction
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
  int stages;  // ring depth: at most kSkStages and the k-blocks per CTA
  int rows_per;  // split-K: output rows reduced (and stored) by each cluster CTA, a power of two >= 4
  int vec_c;     // C rows allow 8-byte stores (16-bit elements, pitch and base multiples of 4 elements)
  const __nv_bfloat16* bias;
  const __nv_bfloat16* resid;
  __nv_bfloat16* C;
  int64_t ldr, ldc;
  const __nv_bfloat16* W;  // [N][K] (row pitch K): L2 prefetch of the slice past the ring
  // Fused decode extras (gemm_skinny_kernel<EPI, true> only; each may be null):
  const float* ln_stats;  // [ln_parts][M][2] (sum, sum of squares) of A's rows: LayerNorm folded in
  const double* ln_sums;  // or [M][2] fp64 totals of the same (one part)
  const float* ln_u;      // [N] row sums of the gamma-scaled weight
  const float* ln_v;      // [N] W . beta + bias (replaces bias)
  int ln_parts;
  float ln_eps, ln_inv_k;
  float* stats_out;       // [ceil(N / 128)][M][2] (sum, sum of squares) of C's stored rows
  __nv_bfloat16* kc;      // KV-cache append of the K and V columns of a fused QKV output:
  __nv_bfloat16* vc;      //   [B = M][H][Tmax][D], position kv_pos0 + *kv_pos
  int kv_C, kv_D, kv_H;
  int64_t kv_tmax, kv_pos0;
  const int64_t* kv_pos;
};

// mean / rstd of row m for the LayerNorm fold, from fp64 totals or fp32 per-part sums.
__device__ __forceinline__ void sk_ln_row(const SkParams& p, int m, float& mean, float& rstd) {
  if (p.ln_sums) {
    const double2 s = *reinterpret_cast<const double2*>(p.ln_sums + 2 * (int64_t)m);
    const double mu = s.x * (double)p.ln_inv_k;
    mean = (float)mu;
    rstd = rsqrtf((float)fmax(s.y * (double)p.ln_inv_k - mu * mu, 0.0) + p.ln_eps);
    return;
  }
  float s1 = 0.f, s2 = 0.f;
  for (int q = 0; q < p.ln_parts; ++q) {
    s1 += p.ln_stats[((int64_t)q * p.M + m) * 2];
    s2 += p.ln_stats[((int64_t)q * p.M + m) * 2 + 1];
  }
  mean = s1 * p.ln_inv_k;
  rstd = rsqrtf(fmaxf(s2 * p.ln_inv_k - mean * mean, 0.f) + p.ln_eps);
}

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
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t sk_cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(local), "r"(rank));
  return out;
}
// Shared memory: [ring: stages x (W slab 16 KB + A rows), reused after the
// main loop as this CTA's fp32 partial [Mp][128]] [split-K receive buffer:
// splits x rows_per x 128 fp32] [barriers]. The ring holds only as many
// stages as a CTA has k-blocks: small footprints let the CTAs of the next
// kernels in the stream become resident early and stream their weight
// slices while this kernel runs.
__host__ __device__ inline int sk_ring_bytes(int Mp, int stages, int splits) {
  const int ring = stages * (128 * BK * 2 + Mp * BK * 2);
  const int part = splits > 1 ? Mp * 128 * 4 : 0;
  return ring > part ? ring : part;
}
__host__ __device__ inline int sk_recv_bytes(int splits, int rows_per) {
  return splits > 1 ? splits * 128 * rows_per * 4 : 0;
}
__host__ __device__ inline int sk_smem_bytes(int Mp, int stages, int splits, int rows_per) {
  return 1024 + sk_ring_bytes(Mp, stages, splits) + sk_recv_bytes(splits, rows_per) + (2 * kSkStages + 2) * 8 + 16;
}
// Dynamic shared memory budget: the 227 KB per CTA less room for the fused
// variant's static arrays (row statistics, LayerNorm mean / rstd).
constexpr int kSkSmemLimit = 232448 - 8192;

template <int EPI, bool kFuse>
__global__ void __launch_bounds__(kSkThreads, 4)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA,
                       const SkParams p) {
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smem_dyn + 1023) & ~(uintptr_t)1023);
  constexpr int kWBytes = 128 * BK * 2;
  const int aBytes = p.Mp * BK * 2;
  const int stages = p.stages;
  uint8_t* ringW = base;
  uint8_t* ringA = base + stages * kWBytes;
  float* part = reinterpret_cast<float*>(base);  // after the main loop
  float* recv = reinterpret_cast<float*>(base + sk_ring_bytes(p.Mp, stages, p.splits));
  uint64_t* bars = (uint64_t*)(base + sk_ring_bytes(p.Mp, stages, p.splits) + sk_recv_bytes(p.splits, p.rows_per));
  uint64_t* full = bars;
  uint64_t* empty = bars + kSkStages;
  uint64_t* done = bars + 2 * kSkStages;
  uint64_t* recv_full = bars + 2 * kSkStages + 1;
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * kSkStages + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const bool clustered = p.splits > 1;
  const int split = clustered ? (int)cluster_ctarank() : 0;
  const int n0 = tile * 128;
  const int kb0 = split * p.kb_per;
  const int kb1 = min(p.nkb, kb0 + p.kb_per);
  const uint32_t tcols = p.Mp <= 32 ? 32u : p.Mp <= 64 ? 64u : p.Mp <= 128 ? 128u : 256u;
  // Split-K: this CTA reduces rows [r_lo, r_lo + r_cnt) of the padded Mp rows.
  const int r_lo = split * p.rows_per;
  const int r_cnt = clustered ? max(0, min(p.rows_per, p.Mp - r_lo)) : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), 1);
    }
    mbar_init(smem_addr(done), 1);
    mbar_init(smem_addr(recv_full), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    // every cluster CTA sends its partial of these rows: splits x 128 x r_cnt fp32
    if (r_cnt > 0) mbar_expect_tx(smem_addr(recv_full), (uint32_t)(p.splits * 128 * r_cnt * 4));
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(tcols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  // Receive barriers of the whole cluster are initialised before any CTA
  // sends (this overlaps the previous kernel: it precedes griddepcontrol.wait).
  if (clustered) {
    cluster_arrive();
    cluster_wait();
  }
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    const uint32_t bytes = (uint32_t)(kWBytes + aBytes);
    // Weights do not depend on earlier kernels: the first ring slots are
    // filled with W before waiting for the previous kernel (programmatic
    // dependent launch), the activation rows after.
    const int pre = min(kb1 - kb0, stages);
    for (int i = 0; i < pre; ++i) {
      const uint32_t fb = smem_addr(&full[i]);
      mbar_expect_tx(fb, bytes);
      tma_load_2d(smem_addr(ringW + i * kWBytes), &tmW, fb, (kb0 + i) * BK, n0);
    }
    pdl_wait();
    pdl_trigger();
    for (int i = 0; i < pre; ++i)
      tma_load_2d(smem_addr(ringA + i * aBytes), &tmA, smem_addr(&full[i]), (kb0 + i) * BK, 0);
    int stage = pre % stages;
    uint32_t phase = pre == stages ? 1u : 0u;
    for (int kb = kb0 + pre; kb < kb1; ++kb) {
      if (!mbar_wait(smem_addr(&empty[stage]), phase ^ 1)) break;
      const uint32_t fb = smem_addr(&full[stage]);
      mbar_expect_tx(fb, bytes);
      tma_load_2d(smem_addr(ringW + stage * kWBytes), &tmW, fb, kb * BK, n0);
      tma_load_2d(smem_addr(ringA + stage * aBytes), &tmA, fb, kb * BK, 0);
      if (++stage == stages) { stage = 0; phase ^= 1; }
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
      if (++stage == stages) { stage = 0; phase ^= 1; }
    }
    tc_commit(smem_addr(done));  // also covers an empty K slice (no MMA issued)
  }
  __syncwarp();
  // The W columns of this CTA's K slice that the pre-filled ring slots do not
  // hold are pulled into L2 before the dependency wait too (warps 2-3, two
  // slab rows per thread; a prefetch is only a hint).
  if (warp >= 2 && p.W) {
    const int kc0 = (kb0 + min(kb1 - kb0, stages)) * BK, kc1 = min(kb1 * BK, p.K);
    if (kc0 < kc1) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = n0 + (warp - 2) * 32 + lane + 64 * h;
        if (row < p.N)
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p.W + (int64_t)row * p.K + kc0),
                       "r"((uint32_t)((kc1 - kc0) * 2))
                       : "memory");
      }
    }
  }
  if (!(warp == 0 && lane == 0)) pdl_wait();

  const int nl = warp * 32 + lane;  // row of the W slab == TMEM lane == output column
  const int n = n0 + nl;
  const bool n_ok = n < p.N;
  const bool has_k = kb1 > kb0;
  const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
  if (!clustered) {
    const bool ok = mbar_wait(smem_addr(done), 0);
    tc_fence_after();
    if constexpr (kFuse) {
      // LayerNorm folded in (the host allows no other extra without split-K):
      // row statistics of all Mp rows into shared memory first.
      __shared__ float ln_ms[kSkMaxM][2];
      const bool lnf = p.ln_stats || p.ln_sums;
      if (lnf) {
        for (int m = threadIdx.x; m < p.M; m += kSkThreads) sk_ln_row(p, m, ln_ms[m][0], ln_ms[m][1]);
      }
      __syncthreads();
      const float un = (lnf && n_ok) ? p.ln_u[n] : 0.f;
      const float vn = (lnf && n_ok) ? p.ln_v[n] : 0.f;
      for (int c = 0; c < p.Mp && ok; c += 32) {
        uint32_t r[32];
        tmem_ld32(lane_base + (uint32_t)c, r);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int m = c + j;
          if (m < p.M && n_ok) {
            float x = __uint_as_float(r[j]);
            if (lnf) x = ln_ms[m][1] * (x - ln_ms[m][0] * un) + vn;
            else if (EPI != GPT_EPI_NONE) x += __bfloat162float(p.bias[n]);
            if (EPI == GPT_EPI_BIAS_GELU) x = gelu_tanh<true>(x);
            if (EPI == GPT_EPI_BIAS_RESIDUAL) x += __bfloat162float(p.resid[(int64_t)m * p.ldr + n]);
            p.C[(int64_t)m * p.ldc + n] = __float2bfloat16_rn(x);
          }
        }
      }
    } else {
      for (int c = 0; c < p.Mp && ok; c += 32) {
        uint32_t r[32];
        tmem_ld32(lane_base + (uint32_t)c, r);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int m = c + j;
          if (m < p.M && n_ok) sk_store<EPI>(p, m, n, __uint_as_float(r[j]));
        }
      }
    }
  } else {
    // Owner epilogue mapping: thread = (row group rs, column group q): rows
    // r_lo + rs, +4, ... and the 4 columns n0 + 4q .. +3, so one warp covers a
    // whole 128-column row segment (float4 reads of the partials, 8-byte
    // stores, row statistics by one warp reduction).
    const int q4 = threadIdx.x & 31;
    const int rs = threadIdx.x >> 5;
    const int nq = n0 + 4 * q4;
    const int ncnt = max(0, min(4, p.N - nq));  // valid columns of this group
    // Bias (or the LayerNorm fold's u / v) of these columns, and the residual
    // of the first row, fetched while the partials are still being produced.
    float b4[4] = {0.f, 0.f, 0.f, 0.f}, u4[4] = {0.f, 0.f, 0.f, 0.f};
    const bool ln = kFuse && (p.ln_stats != nullptr || p.ln_sums != nullptr);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (e < ncnt) {
        if (ln) {
          u4[e] = p.ln_u[nq + e];
          b4[e] = p.ln_v[nq + e];
        } else if (EPI != GPT_EPI_NONE) {
          b4[e] = __bfloat162float(p.bias[nq + e]);
        }
      }
    }
    float rpre[4] = {0.f, 0.f, 0.f, 0.f};
    if (EPI == GPT_EPI_BIAS_RESIDUAL && rs < r_cnt && r_lo + rs < p.M) {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (e < ncnt) rpre[e] = __bfloat162float(p.resid[(int64_t)(r_lo + rs) * p.ldr + nq + e]);
    }
    // LayerNorm fold: mean / rstd of this CTA's output rows from the
    // producer's per-tile partials (published by the barrier before the push).
    __shared__ float ln_ms[64][2];
    if constexpr (kFuse) {
      if (ln && (int)threadIdx.x < r_cnt && r_lo + (int)threadIdx.x < p.M)
        sk_ln_row(p, r_lo + threadIdx.x, ln_ms[threadIdx.x][0], ln_ms[threadIdx.x][1]);
    }
    const bool ok = mbar_wait(smem_addr(done), 0);
    tc_fence_after();
    // Push: the partial goes to shared memory as [Mp][128] (lane == column,
    // conflict-free), then one bulk copy per owner CTA moves its contiguous
    // row block into slot [split] of the owner's receive buffer.
    for (int c = 0; c < p.Mp; c += 32) {
      uint32_t r[32];
      if (ok && has_k) tmem_ld32(lane_base + (uint32_t)c, r);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c + j < p.Mp) part[(c + j) * 128 + nl] = (ok && has_k) ? __uint_as_float(r[j]) : 0.f;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    {
      // lane d of warp 0 sends owner d's row block (copies issued in parallel)
      const int d = threadIdx.x;
      if (d < 32 && d * p.rows_per < p.Mp) {
        const int rows = min(p.rows_per, p.Mp - d * p.rows_per);
        const uint32_t src = smem_addr(part + d * p.rows_per * 128);
        const uint32_t dst = sk_cluster_addr(smem_addr(recv + split * p.rows_per * 128), (uint32_t)d);
        const uint32_t bar = sk_cluster_addr(smem_addr(recv_full), (uint32_t)d);
        asm volatile(
            "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
            "r"(src), "r"((uint32_t)(rows * 128 * 4)), "r"(bar)
            : "memory");
      }
    }
    bool got = true;
    if (r_cnt > 0) {
      got = mbar_wait(smem_addr(recv_full), 0);
    }
    got = __all_sync(0xffffffffu, got);  // warp-uniform: the row statistics use full-warp shuffles
    // Every owner has received its rows, so every bulk copy has finished
    // reading its source: no CTA leaves while a peer still copies from it.
    cluster_arrive();
    if (r_cnt > 0 && got) {
      // KV append target of this column group (k or v part of a fused QKV row;
      // 4 | head_dim keeps the group inside one head).
      __nv_bfloat16* kv_dst = nullptr;
      if constexpr (kFuse) {
        if (p.kc && ncnt > 0 && nq >= p.kv_C) {
          const int idx = nq - p.kv_C;
          const int which = idx / p.kv_C, hd = idx - which * p.kv_C;
          const int h = hd / p.kv_D, d = hd - h * p.kv_D;
          const int64_t kv_pos = p.kv_pos0 + (p.kv_pos ? *p.kv_pos : 0);
          if (kv_pos < p.kv_tmax)
            kv_dst = (which == 0 ? p.kc : p.vc) + ((int64_t)h * p.kv_tmax + kv_pos) * p.kv_D + d;
          else if (q4 == 0 && rs == 0)
            record_device_error(GPT_DEVERR_INDEX);
        }
      }
      const bool vec_c = p.vec_c && ncnt == 4;
#pragma unroll 1
      for (int j = rs; j < r_cnt; j += kSkThreads / 32) {   // warp-uniform
        const int m = r_lo + j;
        if (m >= p.M) break;
        // fixed summation order over the peers (peer 0 first)
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int sidx = 0; sidx < p.splits; ++sidx) {
          const float4 v = *reinterpret_cast<const float4*>(recv + (sidx * p.rows_per + j) * 128 + 4 * q4);
          acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        float radd[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          radd[e] = 0.f;
          if (EPI == GPT_EPI_BIAS_RESIDUAL && e < ncnt)
            radd[e] = j == rs ? rpre[e] : __bfloat162float(p.resid[(int64_t)m * p.ldr + nq + e]);
        }
        float mean = 0.f, rstd = 1.f;
        if (ln) {
          mean = ln_ms[j][0];
          rstd = ln_ms[j][1];
        }
        const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
        __nv_bfloat16 y[4];
        float s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float x = ln ? rstd * (a4[e] - mean * u4[e]) + b4[e] : a4[e] + b4[e];
          if (EPI == GPT_EPI_BIAS_GELU) x = gelu_tanh<true>(x);
          if (EPI == GPT_EPI_BIAS_RESIDUAL) x += radd[e];
          y[e] = __float2bfloat16_rn(x);
          const float yf = e < ncnt ? __bfloat162float(y[e]) : 0.f;
          s1 += yf;
          s2 = fmaf(yf, yf, s2);
        }
        __nv_bfloat16* dst = p.C + (int64_t)m * p.ldc + nq;
        if (vec_c) {
          *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(y);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (e < ncnt) dst[e] = y[e];
        }
        if constexpr (kFuse) {
          if (kv_dst) {
            __nv_bfloat16* kd = kv_dst + (int64_t)m * p.kv_H * p.kv_tmax * p.kv_D;
            if (ncnt == 4) {
              *reinterpret_cast<uint2*>(kd) = *reinterpret_cast<const uint2*>(y);
            } else {
              for (int e = 0; e < ncnt; ++e) kd[e] = y[e];
            }
          }
          if (p.stats_out) {  // one warp holds the whole 128-column segment of row m
            s1 = warp_sum(s1);
            s2 = warp_sum(s2);
            if (q4 == 0) {
              float* sd = p.stats_out + ((int64_t)tile * p.M + m) * 2;
              sd[0] = s1;
              sd[1] = s2;
            }
          }
        }
      }
    }
    cluster_wait();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols));
  }
}

struct SkPlan {
  int Mp, tiles, nkb, kb_per, splits, stages, rows_per;
};

// Splits: enough CTAs for about two per three SMs, at most the cluster size
// limit, never an empty K slice. Each cluster CTA then reduces rows_per output rows
// (a power of two, at least 4, splits x rows_per >= Mp); the ring gets as
// many stages as fit beside the receive buffer.
inline SkPlan sk_plan(int64_t M, int64_t N, int64_t K, int sms, int max_splits, int min_splits = 1,
                      int max_rows_per = kSkMaxM) {
  SkPlan pl;
  pl.Mp = (int)(((M + 15) / 16) * 16);
  pl.tiles = (int)((N + 127) / 128);
  pl.nkb = (int)((K + BK - 1) / BK);
  // About two CTAs for every three SMs: measured on B200 (M = 64, GPT-2
  // shapes, CUDA-graph replay) this beats one or two per SM, since the next
  // kernel's CTAs need room to become resident while this one runs.
  int want = (2 * sms / 3 + pl.tiles - 1) / pl.tiles;
  const int min_rows = (pl.Mp + max_rows_per - 1) / max_rows_per;
  if (want < min_splits) want = min_splits;
  if (want < min_rows) want = min_rows;
  if (want > max_splits) want = max_splits;
  if (want > pl.nkb) want = pl.nkb;
  if (want < 1) want = 1;
  while (true) {
    pl.kb_per = (pl.nkb + want - 1) / want;
    pl.splits = (pl.nkb + pl.kb_per - 1) / pl.kb_per;
    pl.rows_per = 4;
    while (pl.splits > 1 && pl.rows_per * pl.splits < pl.Mp) pl.rows_per *= 2;
    pl.stages = pl.kb_per < kSkStages ? pl.kb_per : kSkStages;
    while (pl.stages > 1 && sk_smem_bytes(pl.Mp, pl.stages, pl.splits, pl.rows_per) > kSkSmemLimit) --pl.stages;
    if (sk_smem_bytes(pl.Mp, pl.stages, pl.splits, pl.rows_per) <= kSkSmemLimit || want == 1) break;
    want = want > 2 ? want / 2 : 1;
  }
  return pl;
}

template <int EPI, bool kFuse>
static int sk_launch(const CUtensorMap& tw, const CUtensorMap& ta, const SkParams& p, int tiles, int smem,
                     cudaStream_t st) {
  auto kern = gemm_skinny_kernel<EPI, kFuse>;
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
template <int EPI, bool kFuse>
static int sk_setup(int* max_splits) {
  static int cached[64] = {0};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(GPT_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> g(mu);
  if (cached[dev] == 0) {
    auto kern = gemm_skinny_kernel<EPI, kFuse>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSkSmemLimit);
    if (e != cudaSuccess) return fail(GPT_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    // Clusters above 8 CTAs are non-portable; they are used only when the
    // attribute is accepted and a 16-CTA cluster of the largest footprint fits.
    int ms = 8;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, kSkMaxSplits, 1);
      cfg.blockDim = dim3(kSkThreads, 1, 1);
      cfg.dynamicSmemBytes = (size_t)kSkSmemLimit;
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

template <int EPI, bool kFuse>
static int gemm_skinny_epi(const void* A, int64_t lda, const void* W, const SkParams& p0, int64_t M, int64_t N,
                           int64_t K, cudaStream_t st) {
  int max_splits = 8;
  int s = sk_setup<EPI, kFuse>(&max_splits);
  if (s) return s;
  int sms = device_sm_count();
  if (sms <= 0) return fail(GPT_ERR_CUDA, "no CUDA device");
  // Output statistics and the KV append live in the split-K owner epilogue
  // (at least 2 splits, at most 64 rows per owner CTA).
  const bool owner_extras = kFuse && (p0.stats_out || p0.kc);
  SkPlan pl = sk_plan(M, N, K, sms, max_splits, owner_extras ? 2 : 1, kFuse ? 64 : kSkMaxM);
  if (owner_extras && pl.splits < 2)
    return fail(GPT_ERR_UNSUPPORTED, "gpt_gemm_fused: row statistics / KV append need K >= %d", 2 * BK);
  CUtensorMap tw, ta;
  s = make_map(&tw, W, N, K, K, 128);
  if (s) return s;
  s = make_map(&ta, A, M, K, lda, pl.Mp);
  if (s) return s;
  SkParams p = p0;
  p.W = (const __nv_bfloat16*)W;
  p.Mp = pl.Mp;
  p.nkb = pl.nkb;
  p.kb_per = pl.kb_per;
  p.splits = pl.splits;
  p.stages = pl.stages;
  p.rows_per = pl.rows_per;
  return sk_launch<EPI, kFuse>(tw, ta, p, pl.tiles, sk_smem_bytes(pl.Mp, p.stages, p.splits, p.rows_per), st);
}

// Serves bf16 requests with M <= kSkMaxM rows.
int gemm_skinny(const void* A, int64_t lda, const void* W, const void* bias, const void* R, int64_t ldr, void* C,
                int64_t ldc, int64_t M, int64_t N, int64_t K, int epi, cudaStream_t st) {
  SkParams p = {};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.bias = (const __nv_bfloat16*)bias;
  p.resid = (const __nv_bfloat16*)R;
  p.C = (__nv_bfloat16*)C;
  p.ldr = ldr;
  p.ldc = ldc;
  p.vec_c = aligned(C, 8) && ldc % 4 == 0;
  switch (epi) {
    case GPT_EPI_NONE: return gemm_skinny_epi<GPT_EPI_NONE, false>(A, lda, W, p, M, N, K, st);
    case GPT_EPI_BIAS: return gemm_skinny_epi<GPT_EPI_BIAS, false>(A, lda, W, p, M, N, K, st);
    case GPT_EPI_BIAS_GELU: return gemm_skinny_epi<GPT_EPI_BIAS_GELU, false>(A, lda, W, p, M, N, K, st);
    default: return gemm_skinny_epi<GPT_EPI_BIAS_RESIDUAL, false>(A, lda, W, p, M, N, K, st);
  }
}

// Few-row GEMM with the fused decode extras (LayerNorm fold, output row
// statistics, KV append); the caller has validated the arguments.
int gemm_skinny_fused(const void* A, int64_t lda, const void* W, const void* bias, const void* R, int64_t ldr,
                      void* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int epi, const gpt_gemm_fusion& f,
                      cudaStream_t st) {
  SkParams p = {};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.bias = (const __nv_bfloat16*)bias;
  p.resid = (const __nv_bfloat16*)R;
  p.C = (__nv_bfloat16*)C;
  p.ldr = ldr;
  p.ldc = ldc;
  p.vec_c = aligned(C, 8) && ldc % 4 == 0;
  p.ln_stats = f.ln_stats;
  p.ln_sums = f.ln_sums;
  p.ln_u = f.ln_u;
  p.ln_v = f.ln_v;
  p.ln_parts = (int)f.ln_parts;
  p.ln_eps = f.ln_eps;
  p.ln_inv_k = 1.0f / (float)K;
  p.stats_out = f.row_stats;
  p.kc = (__nv_bfloat16*)f.k_cache;
  p.vc = (__nv_bfloat16*)f.v_cache;
  p.kv_C = (int)(f.kv_heads * f.kv_dim);
  p.kv_D = (int)f.kv_dim;
  p.kv_H = (int)f.kv_heads;
  p.kv_tmax = f.kv_tmax;
  p.kv_pos0 = f.kv_pos0;
  p.kv_pos = f.kv_pos_dev;
  switch (epi) {
    case GPT_EPI_NONE: return gemm_skinny_epi<GPT_EPI_NONE, true>(A, lda, W, p, M, N, K, st);
    case GPT_EPI_BIAS: return gemm_skinny_epi<GPT_EPI_BIAS, true>(A, lda, W, p, M, N, K, st);
    case GPT_EPI_BIAS_GELU: return gemm_skinny_epi<GPT_EPI_BIAS_GELU, true>(A, lda, W, p, M, N, K, st);
    default: return gemm_skinny_epi<GPT_EPI_BIAS_RESIDUAL, true>(A, lda, W, p, M, N, K, st);
  }
}

}  // namespace tc
}  // namespace gpt
