// One decode step (all transformer blocks for one new token per sequence)
// as a single persistent kernel: GPT-2 blocks, bf16, head_dim 64, up to 64
// sequences per GPU. The reference has no decode path (it re-runs the full
// forward per token, cutile_gpt/models/gpt.py:204-206).
//
// Why one kernel: at B <= 64 rows every GEMM of a block moves only 1-5 MB
// of weights, so a kernel per op is bound by launch and pipeline latency
// (~8 us each, 8 per block). Here every SM runs one CTA for the whole step:
//   warp 4 lane 0   streams this CTA's weight slabs (128 rows x 64 k, one
//                   TMA box each) for every GEMM of every block, in order,
//                   through a 10-slot shared-memory ring — before the
//                   programmatic-dependent-launch wait, so the first blocks'
//                   weights arrive while the previous kernel drains;
//   warps 0-3       run the phases of each block, separated by grid
//                   barriers:
//     R1  x += W2-output of the previous block (or the embedding), LN1 stats
//     A   qkv  += LN1(x) W_qkvᵀ          (unit = 128 weight rows x 64 k)
//     B   attention per (sequence, head): bias, K/V append to the cache,
//         online softmax over the cached positions -> att
//     C   proj += att W_projᵀ
//     R2  x += proj + b_proj, LN2 stats
//     D   fc   += LN2(x) W_fcᵀ
//     E   fc2  += gelu(fc + b_fc) W_projᵀ
//   and after the last block x += fc2 + b and h = ln_f(x) (bf16, [B, C]),
//   which the lm_head GEMM reads.
// GEMM units are tcgen05.mma with the weight slab as the 128-row operand and
// the activation rows (padded to Mp = 32 or 64) as the N side, fp32 in TMEM;
// partial sums are added into fp32 accumulators [N][Mp] with vector
// red.global.add (split over K across CTAs). Each accumulator is cleared by
// the whole grid (coalesced stores) in a phase after the one that consumed
// it, so the workspace is back to zero before its next use in the step.
// Data written by other CTAs is read with ld.global.cg (L2), never from L1.
// Every wait is bounded; on expiry the kernel records GPT_DEVERR_TIMEOUT.
#include <stdlib.h>
#include <vector>

#include "common.cuh"

namespace gpt {
namespace fused {

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
using tc::tmem_ld32;

constexpr int kCompute = 128;            // 4 compute warps
constexpr int kThreads = kCompute + 32;  // + producer warp
constexpr int kSlots = 10;               // weight ring depth (16 KB each)
constexpr int kSlotBytes = 128 * 64 * 2;
constexpr int kMaxMp = 64;
constexpr int kABytes = kMaxMp * 64 * 2;  // activation tile, 8 KB
constexpr int kBatch = 4;                 // units of one phase issued together per CTA
constexpr int kSmem = 1024 + kSlots * kSlotBytes + kBatch * kABytes + 256;
constexpr int kPhases = 4;               // GEMM phases per block: qkv, proj, fc, proj2
constexpr uint64_t kWaitNs = 2000000000ull;

struct LayerW {  // device pointers of one block (nn.Linear [out, in] weights)
  const __nv_bfloat16 *ln1_w, *ln1_b, *b_qkv, *b_proj, *ln2_w, *ln2_b, *b_fc, *b_proj2;
};

struct Plan {  // built on the host once per model, copied to device memory
  CUtensorMap maps[1];  // [L][4] weight maps follow (64-byte aligned)
};

struct Params {
  const CUtensorMap* maps;  // [L * 4]
  const LayerW* layers;     // [L]
  int L, C, H, B, Mp, Tmax, n_pos, vocab;
  float eps, scale_log2;
  const int64_t* tok;
  const int64_t* pos_dev;
  const __nv_bfloat16 *wte, *wpe, *lnf_w, *lnf_b;
  __nv_bfloat16* cache;     // [L][2][B][H][Tmax][64]
  __nv_bfloat16* h_out;     // [B][C]
  // workspace
  __nv_bfloat16 *x, *att;   // [Mp][C]
  float *acc_qkv, *acc_proj, *acc_fc, *acc_fc2;  // [N][Mp]
  float* stats;             // [2][Mp][2] (mean, rstd) for LN1 / LN2
  unsigned long long* bar;  // grid barrier arrivals (monotonic)
  unsigned long long* trace;  // optional: %globaltimer at each phase boundary (CTA 0), or null
};

__device__ __forceinline__ unsigned long long ld_acq64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void compute_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Grid barrier among the compute warps of all CTAs. Arrival k of a launch
// returns once the counter reaches the next multiple of gridDim.x; the
// counter never resets, so no CTA has to observe a separate generation word.
__device__ bool grid_sync(unsigned long long* bar) {
  __threadfence();
  compute_bar();
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    unsigned long long old;
    asm volatile("atom.add.release.gpu.global.u64 %0, [%1], 1;" : "=l"(old) : "l"(bar) : "memory");
    const unsigned long long target = (old / gridDim.x + 1) * gridDim.x;
    int ok = 1;
    if (ld_acq64(bar) < target) {
      const uint64_t t0 = global_timer_ns();
      while (ld_acq64(bar) < target) {
        if (global_timer_ns() - t0 > kWaitNs) {
          record_device_error(GPT_DEVERR_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  compute_bar();
  return s_ok != 0;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[w] = v;
  compute_bar();
  float s = red[0] + red[1] + red[2] + red[3];
  compute_bar();
  return s;
}

// ---- unit bookkeeping shared by the producer and the compute warps
struct Gemm {
  int N, K;
};
__device__ __forceinline__ Gemm gemm_of(int phase, int C) {
  switch (phase) {
    case 0: return {3 * C, C};
    case 1: return {C, C};
    case 2: return {4 * C, C};
    default: return {C, 4 * C};
  }
}
__device__ __forceinline__ int units_of(const Gemm& g) { return (g.N / 128) * (g.K / 64); }

// Activation tile for one unit: rows m < Mp, 64 k values starting at k0,
// written as bf16 in the 128B-swizzled K-major layout the MMA reads.
template <int SRC>  // 0: LN(x) with stats, 1: att, 2: gelu(acc_fc + b)
__device__ void build_a(const Params& p, uint8_t* sA, int k0, const float* stats, const __nv_bfloat16* g,
                        const __nv_bfloat16* bvec) {
  const int tid = threadIdx.x;
  if (SRC == 2) {
    // acc_fc is [k][Mp]: each thread takes two adjacent k and four rows m
    // (two 16-byte loads) and writes bf16 pairs.
    for (int c = tid; c < 32 * (p.Mp / 4); c += kCompute) {
      const int kl = (c & 31) * 2, m0 = (c >> 5) * 4;
      const int kk = k0 + kl;
      const float4 a0 = __ldcg(reinterpret_cast<const float4*>(p.acc_fc + (int64_t)kk * p.Mp + m0));
      const float4 a1 = __ldcg(reinterpret_cast<const float4*>(p.acc_fc + (int64_t)(kk + 1) * p.Mp + m0));
      const float b0 = __bfloat162float(bvec[kk]), b1 = __bfloat162float(bvec[kk + 1]);
      const float v0[4] = {a0.x, a0.y, a0.z, a0.w}, v1[4] = {a1.x, a1.y, a1.z, a1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int m = m0 + i;
        const bool real = m < p.B;
        __nv_bfloat162 t = __floats2bfloat162_rn(real ? gelu_tanh<true>(v0[i] + b0) : 0.f,
                                                 real ? gelu_tanh<true>(v1[i] + b1) : 0.f);
        *reinterpret_cast<__nv_bfloat162*>(sA + m * 128 + (((kl >> 3) ^ (m & 7)) << 4) + (kl & 7) * 2) = t;
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    return;
  }
  for (int c = tid; c < p.Mp * 8; c += kCompute) {   // 16-byte chunks: row m, k-chunk kc
    const int m = c >> 3, kc = c & 7;
    const int kk = k0 + kc * 8;
    float v[8];
    if (m >= p.B) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    } else if (SRC == 0) {
      const float mean = __ldcg(stats + m * 2), rstd = __ldcg(stats + m * 2 + 1);
      const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(p.x + (int64_t)m * p.C + kk));
      const uint4 graw = *reinterpret_cast<const uint4*>(g + kk);
      const uint4 braw = *reinterpret_cast<const uint4*>(bvec + kk);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
      const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&graw);
      const __nv_bfloat16* be = reinterpret_cast<const __nv_bfloat16*>(&braw);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        v[i] = (__bfloat162float(e[i]) - mean) * rstd * __bfloat162float(ge[i]) + __bfloat162float(be[i]);
    } else {
      const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(p.att + (int64_t)m * p.C + kk));
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(e[i]);
    }
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 t = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&t);
    }
    *reinterpret_cast<uint4*>(sA + m * 128 + ((kc ^ (m & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor core
}

// Zeroes this CTA's share of a float array (16-byte stores spread over the grid).
__device__ __forceinline__ void zero_share(float* ptr, int64_t n) {
  const int64_t n4 = n / 4;
  for (int64_t i = (int64_t)blockIdx.x * kCompute + threadIdx.x; i < n4; i += (int64_t)gridDim.x * kCompute)
    __stcg(reinterpret_cast<float4*>(ptr) + i, make_float4(0.f, 0.f, 0.f, 0.f));
}

struct RingState {
  int k = 0;       // units consumed by the compute warps
  int mma = 0;     // MMA completions waited for
};

// One GEMM phase of block l; partial sums -> acc. Each CTA owns a
// contiguous run of units (n-tile major, k-block minor), so consecutive
// k-blocks of one weight slab accumulate in TMEM and are reduced into acc
// once. Up to kBatch units are built, issued back to back and reduced
// together, so a phase costs about one round trip.
template <int SRC>
__device__ bool gemm_phase(const Params& p, int l, int phase, uint8_t* ring, uint8_t* sA, uint64_t* full,
                           uint64_t* empty, uint64_t* mma_done, uint32_t tmem, RingState& rs, float* acc,
                           const float* stats, const __nv_bfloat16* g, const __nv_bfloat16* bvec) {
  const Gemm gm = gemm_of(phase, p.C);
  const int kb_n = gm.K / 64;
  const int U = units_of(gm);
  const int tid = threadIdx.x, warp = tid >> 5;
  bool ok = true;
  // kind::f16, D fp32, A = weight slab (128 rows, K-major), B = activation rows (Mp, K-major)
  const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.Mp >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
  const int u_begin = (int)((int64_t)blockIdx.x * U / gridDim.x);
  const int u_end = (int)((int64_t)(blockIdx.x + 1) * U / gridDim.x);
  for (int u0 = u_begin; u0 < u_end; u0 += kBatch) {
    const int nb = min(kBatch, u_end - u0);
    for (int i = 0; i < nb; ++i) build_a<SRC>(p, sA + i * kABytes, ((u0 + i) % kb_n) * 64, stats, g, bvec);
    tc_fence_before();
    compute_bar();
    if (tid == 0) {
      int grp = -1, prev_nt = -1;
      for (int i = 0; i < nb; ++i) {
        const int nt = (u0 + i) / kb_n;
        const bool first = nt != prev_nt;
        if (first) ++grp;
        prev_nt = nt;
        const int k = rs.k + i, slot = k % kSlots;
        if (!mbar_wait(smem_addr(&full[slot]), (uint32_t)((k / kSlots) & 1))) ok = false;
        tc_fence_after();
        const uint64_t wd = desc_sw128(smem_addr(ring + slot * kSlotBytes));
        const uint64_t ad = desc_sw128(smem_addr(sA + i * kABytes));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma(tmem + (uint32_t)(grp * 64), wd + (uint64_t)(2 * kk), ad + (uint64_t)(2 * kk), idesc,
                 (!first || kk > 0) ? 1u : 0u);
        tc_commit(smem_addr(&empty[slot]));
      }
      tc_commit(smem_addr(mma_done));
    }
    rs.k += nb;
    if (!mbar_wait(smem_addr(mma_done), (uint32_t)(rs.mma & 1))) ok = false;
    ++rs.mma;
    tc_fence_after();
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    int grp = -1, prev_nt = -1;
    for (int i = 0; i < nb; ++i) {
      const int nt = (u0 + i) / kb_n;
      if (nt == prev_nt) continue;   // reduce each slab group once
      prev_nt = nt;
      ++grp;
      // thread tid owns weight row n; red-add its Mp partial sums (vectors of 4)
      float* dst = acc + (int64_t)(nt * 128 + tid) * p.Mp;
      for (int c = 0; c < p.Mp; c += 32) {
        uint32_t r[32];
        tmem_ld32(lane_base + (uint32_t)(grp * 64 + c), r);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          if (c + j < p.B)
            asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + c + j),
                         "f"(__uint_as_float(r[j])), "f"(__uint_as_float(r[j + 1])), "f"(__uint_as_float(r[j + 2])),
                         "f"(__uint_as_float(r[j + 3]))
                         : "memory");
        }
      }
    }
    tc_fence_before();
    compute_bar();  // sA and TMEM are reused by the next batch
  }
  return ok;
}

// Row phase: x[m] (+)= addend, LN stats (the consumed accumulators are
// cleared later by zero_share, off this phase's critical path).
// mode 0: embedding; 1: + acc_fc2 + b_proj2 of block l-1; 2: + acc_proj + b_proj of block l;
// 3: final (as 1, then h_out = ln_f(x)). Thread t handles columns t + 128 i.
constexpr int kMaxPerThread = 16;  // n_embd <= 2048
__device__ void row_phase(const Params& p, int mode, int l, float* stats, float* red) {
  const int tid = threadIdx.x;
  const int64_t pos = *p.pos_dev;
  const int npt = p.C / kCompute;
  for (int m = blockIdx.x; m < p.Mp; m += gridDim.x) {
    const bool real = m < p.B;
    float v[kMaxPerThread];
    float s = 0.f;
    if (real) {
      if (mode == 0) {
        const int64_t id = p.tok[m];
        const bool ok = id >= 0 && id < p.vocab && pos >= 0 && pos < p.n_pos;
        if (!ok && tid == 0) record_device_error(GPT_DEVERR_INDEX);
#pragma unroll
        for (int i = 0; i < kMaxPerThread; ++i)
          if (i < npt) {
            const int n = tid + i * kCompute;
            v[i] = ok ? __bfloat162float(p.wte[id * p.C + n]) + __bfloat162float(p.wpe[pos * p.C + n]) : 0.f;
          }
      } else {
        const float* acc = mode == 2 ? p.acc_proj : p.acc_fc2;
        const __nv_bfloat16* bias = mode == 2 ? p.layers[l].b_proj : p.layers[l - 1].b_proj2;
        float a[kMaxPerThread];
#pragma unroll
        for (int i = 0; i < kMaxPerThread; ++i)   // all loads first
          if (i < npt) {
            const int n = tid + i * kCompute;
            v[i] = __bfloat162float(__ldcg(p.x + (int64_t)m * p.C + n));
            a[i] = __ldcg(acc + (int64_t)n * p.Mp + m) + __bfloat162float(bias[n]);
          }
#pragma unroll
        for (int i = 0; i < kMaxPerThread; ++i)
          if (i < npt) v[i] += a[i];
      }
#pragma unroll
      for (int i = 0; i < kMaxPerThread; ++i)
        if (i < npt) {
          // the residual stream is bf16, as in the layer-by-layer path
          const __nv_bfloat16 xb = __float2bfloat16_rn(v[i]);
          p.x[(int64_t)m * p.C + tid + i * kCompute] = xb;
          v[i] = __bfloat162float(xb);
          s += v[i];
        }
    }
    const float mean = block_sum(s, red) / (float)p.C;
    float q = 0.f;
    if (real) {
#pragma unroll
      for (int i = 0; i < kMaxPerThread; ++i)
        if (i < npt) q += (v[i] - mean) * (v[i] - mean);
    }
    const float rstd = rsqrtf(block_sum(q, red) / (float)p.C + p.eps);
    if (mode == 3) {
      if (real) {
#pragma unroll
        for (int i = 0; i < kMaxPerThread; ++i)
          if (i < npt) {
            const int n = tid + i * kCompute;
            p.h_out[(int64_t)m * p.C + n] = __float2bfloat16_rn((v[i] - mean) * rstd * __bfloat162float(p.lnf_w[n]) +
                                                                __bfloat162float(p.lnf_b[n]));
          }
      }
    } else if (tid == 0) {
      stats[m * 2] = mean;
      stats[m * 2 + 1] = rstd;
    }
  }
}

// Attention, one warp per (sequence b, head h): bias, K/V of the new
// position appended to the cache, online softmax over positions 0..pos
// (cached keys from global memory, the new one from registers), output row
// -> att. 8 lanes per key (16 bytes = 8 dims each), 4 keys per warp step,
// 8 steps in flight; the running max / sum are updated once per 8 keys.
__device__ void attention_phase(const Params& p, int l, float* sq_all, float* sk_all) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sub = lane & 7, grp = lane >> 3;
  const int64_t pos = *p.pos_dev;
  const int C = p.C;
  const int kmax = (int)min((int64_t)p.Tmax, pos);   // cached positions before the new one
  const __nv_bfloat16* bq = p.layers[l].b_qkv;
  float* sq = sq_all + warp * 64;
  float* sk = sk_all + warp * 128;   // new key (64) and value (64)
  for (int u = blockIdx.x * 4 + warp; u < p.B * p.H; u += gridDim.x * 4) {   // warp-uniform
    const int b = u / p.H, h = u % p.H;
    __nv_bfloat16* kc = p.cache + ((((int64_t)l * 2 + 0) * p.B + b) * p.H + h) * (int64_t)p.Tmax * 64;
    __nv_bfloat16* vc = p.cache + ((((int64_t)l * 2 + 1) * p.B + b) * p.H + h) * (int64_t)p.Tmax * 64;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int d = lane + 32 * half;
      float* aq = p.acc_qkv + (int64_t)(h * 64 + d) * p.Mp + b;
      float* ak = p.acc_qkv + (int64_t)(C + h * 64 + d) * p.Mp + b;
      float* av = p.acc_qkv + (int64_t)(2 * C + h * 64 + d) * p.Mp + b;
      const float q = __ldcg(aq) + __bfloat162float(bq[h * 64 + d]);
      const float k = __ldcg(ak) + __bfloat162float(bq[C + h * 64 + d]);
      const float v = __ldcg(av) + __bfloat162float(bq[2 * C + h * 64 + d]);
      const __nv_bfloat16 kb = __float2bfloat16_rn(k), vb = __float2bfloat16_rn(v);
      sq[d] = __bfloat162float(__float2bfloat16_rn(q)) * p.scale_log2;   // as the bf16 QKV output
      sk[d] = __bfloat162float(kb);
      sk[64 + d] = __bfloat162float(vb);
      if (pos < p.Tmax) {
        kc[pos * 64 + d] = kb;
        vc[pos * 64 + d] = vb;
      }
    }
    __syncwarp();
    float qv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) qv[i] = sq[sub * 8 + i];
    float m_run = -INFINITY, l_run = 0.f, acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int jb = 0; jb < kmax; jb += 32) {   // warp-uniform bound
      uint4 kr[8], vr[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int j = jb + grp + 4 * t;
        kr[t] = vr[t] = make_uint4(0, 0, 0, 0);
        if (j < kmax) {
          kr[t] = __ldcg(reinterpret_cast<const uint4*>(kc + (int64_t)j * 64 + sub * 8));
          vr[t] = __ldcg(reinterpret_cast<const uint4*>(vc + (int64_t)j * 64 + sub * 8));
        }
      }
      float dots[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const __nv_bfloat16* ke = reinterpret_cast<const __nv_bfloat16*>(&kr[t]);
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) dot = fmaf(qv[i], __bfloat162float(ke[i]), dot);
        dots[t] = dot;
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int t = 0; t < 8; ++t) dots[t] += __shfl_xor_sync(0xffffffffu, dots[t], o);
      float mn = m_run;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        if (jb + grp + 4 * t >= kmax) dots[t] = -INFINITY;
        mn = fmaxf(mn, dots[t]);
      }
      if (mn != -INFINITY) {
        const float a = exp2f(m_run - mn);
        l_run *= a;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] *= a;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const float pe = exp2f(dots[t] - mn);
          const __nv_bfloat16* ve = reinterpret_cast<const __nv_bfloat16*>(&vr[t]);
          l_run += pe;
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = fmaf(pe, __bfloat162float(ve[i]), acc[i]);
        }
        m_run = mn;
      }
    }
    {  // the new position (key group 0 only)
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) dot = fmaf(qv[i], sk[sub * 8 + i], dot);
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      dot += __shfl_xor_sync(0xffffffffu, dot, 4);
      if (grp == 0) {
        const float mn = fmaxf(m_run, dot);
        const float a = exp2f(m_run - mn), pe = exp2f(dot - mn);
        l_run = l_run * a + pe;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(acc[i], a, pe * sk[64 + sub * 8 + i]);
        m_run = mn;
      }
    }
    // merge the 4 key groups of the warp
#pragma unroll
    for (int o = 8; o < 32; o <<= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, m_run, o), lo = __shfl_xor_sync(0xffffffffu, l_run, o);
      const float mn = fmaxf(m_run, mo);
      const float a = mn == -INFINITY ? 0.f : exp2f(m_run - mn), bo = mn == -INFINITY ? 0.f : exp2f(mo - mn);
      l_run = l_run * a + lo * bo;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = acc[i] * a + __shfl_xor_sync(0xffffffffu, acc[i], o) * bo;
      m_run = mn;
    }
    if (grp == 0) {
      const float inv = 1.f / l_run;
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 t2 = __floats2bfloat162_rn(acc[2 * i] * inv, acc[2 * i + 1] * inv);
        w[i] = *reinterpret_cast<uint32_t*>(&t2);
      }
      *reinterpret_cast<uint4*>(p.att + (int64_t)b * C + h * 64 + sub * 8) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    __syncwarp();   // sq / sk are rewritten by the next unit
  }
}

__global__ void __launch_bounds__(kThreads, 1) decode_fused_kernel(const Params p) {
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smem_dyn + 1023) & ~(uintptr_t)1023);
  uint8_t* ring = base;
  uint8_t* sA = ring + kSlots * kSlotBytes;   // kBatch activation tiles
  uint64_t* bars = (uint64_t*)(sA + kBatch * kABytes);
  uint64_t* full = bars;                  // [kSlots]
  uint64_t* empty = bars + kSlots;        // [kSlots]
  uint64_t* mma_done = bars + 2 * kSlots;
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * kSlots + 1);
  __shared__ float red[8];
  __shared__ float sq[4 * 64], skv[4 * 128];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t tcols = 256u;   // kBatch units x up to 64 columns
  if (tid == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(smem_addr(&full[i]), 1);
      mbar_init(smem_addr(&empty[i]), 1);
    }
    mbar_init(smem_addr(mma_done), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(tcols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------ weight stream (independent of earlier kernels)
    if (lane == 0) {
      int k = 0;
      for (int l = 0; l < p.L; ++l) {
        for (int ph = 0; ph < kPhases; ++ph) {
          const CUtensorMap* map = p.maps + l * kPhases + ph;
          const Gemm gm = gemm_of(ph, p.C);
          const int kb_n = gm.K / 64;
          const int U = units_of(gm);
          const int u_end = (int)((int64_t)(blockIdx.x + 1) * U / gridDim.x);
          for (int u = (int)((int64_t)blockIdx.x * U / gridDim.x); u < u_end; ++u, ++k) {
            const int slot = k % kSlots;
            if (k >= kSlots && !mbar_wait(smem_addr(&empty[slot]), (uint32_t)(((k / kSlots) - 1) & 1))) break;
            const uint32_t fb = smem_addr(&full[slot]);
            mbar_expect_tx(fb, kSlotBytes);
            tma_load_2d(smem_addr(ring + slot * kSlotBytes), map, fb, (u % kb_n) * 64, (u / kb_n) * 128);
          }
        }
      }
    }
    pdl_trigger();
  } else {
    pdl_wait();
    pdl_trigger();
    RingState rs;
    bool ok = true;
    int ti = 0;
    auto mark = [&]() {
      if (p.trace && blockIdx.x == 0 && tid == 0) p.trace[ti] = global_timer_ns();
      ++ti;
    };
    mark();
    float* stats1 = p.stats;
    float* stats2 = p.stats + 2 * kMaxMp;
    for (int l = 0; l < p.L && ok; ++l) {
      const LayerW& lw = p.layers[l];
      row_phase(p, l == 0 ? 0 : 1, l, stats1, red);
      mark();
      ok = ok && grid_sync(p.bar);
      mark();
      zero_share(p.acc_fc, (int64_t)4 * p.C * p.Mp);    // consumed by E of the previous block
      zero_share(p.acc_fc2, (int64_t)p.C * p.Mp);       // consumed by R1 above
      ok = gemm_phase<0>(p, l, 0, ring, sA, full, empty, mma_done, tmem, rs, p.acc_qkv, stats1, lw.ln1_w, lw.ln1_b) && ok;
      mark();
      ok = ok && grid_sync(p.bar);
      mark();
      attention_phase(p, l, sq, skv);
      mark();
      ok = ok && grid_sync(p.bar);
      mark();
      zero_share(p.acc_qkv, (int64_t)3 * p.C * p.Mp);   // consumed by the attention phase
      ok = gemm_phase<1>(p, l, 1, ring, sA, full, empty, mma_done, tmem, rs, p.acc_proj, nullptr, nullptr, nullptr) && ok;
      mark();
      ok = ok && grid_sync(p.bar);
      mark();
      row_phase(p, 2, l, stats2, red);
      mark();
      ok = ok && grid_sync(p.bar);
      mark();
      zero_share(p.acc_proj, (int64_t)p.C * p.Mp);      // consumed by R2
      ok = gemm_phase<0>(p, l, 2, ring, sA, full, empty, mma_done, tmem, rs, p.acc_fc, stats2, lw.ln2_w, lw.ln2_b) && ok;
      mark();
      ok = ok && grid_sync(p.bar);
      mark();
      ok = gemm_phase<2>(p, l, 3, ring, sA, full, empty, mma_done, tmem, rs, p.acc_fc2, nullptr, nullptr, lw.b_fc) && ok;
      mark();
      ok = ok && grid_sync(p.bar);
      mark();
    }
    if (ok) row_phase(p, 3, p.L, nullptr, red);
    mark();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols));
  }
}

// ---- host side
constexpr int kTraceSlots = 2 + 14 * 64;   // up to 64 blocks
inline int64_t ws_bytes(int64_t C, int Mp) {
  int64_t b = 0;
  b += 2 * (int64_t)Mp * C * 2;          // x, att
  b += (3 + 1 + 4 + 1) * C * (int64_t)Mp * 4;  // accumulators
  b += 4 * kMaxMp * 4;                   // stats
  b += 256;                              // barrier counter (own 256-byte line)
  b += kTraceSlots * 8;                  // optional phase trace
  return (b + 255) / 256 * 256 + 256;
}

}  // namespace fused
}  // namespace gpt

extern "C" {

int64_t gpt_decode_fused_plan_bytes(int64_t L) {
  return L > 0 ? L * gpt::fused::kPhases * (int64_t)sizeof(CUtensorMap) + L * (int64_t)sizeof(gpt::fused::LayerW) + 128 : 0;
}

int64_t gpt_decode_fused_workspace_bytes(int64_t B, int64_t C) {
  if (B <= 0 || B > gpt::fused::kMaxMp || C <= 0) return 0;
  const int Mp = B <= 32 ? 32 : 64;
  return gpt::fused::ws_bytes(C, Mp);
}

int gpt_decode_fused_plan(void* plan, int64_t plan_bytes, const void* const* ptrs, int64_t L, int64_t C) {
  using namespace gpt::fused;
  GPT_CHECK_SHAPE(L > 0 && C > 0 && C % 128 == 0 && plan_bytes >= gpt_decode_fused_plan_bytes(L),
                  "gpt_decode_fused_plan: needs n_embd % 128 == 0 and a plan buffer of %lld bytes",
                  (long long)gpt_decode_fused_plan_bytes(L));
  GPT_CHECK_ARG(plan && ptrs, "gpt_decode_fused_plan: null pointer");
  GPT_CHECK_ALIGN(gpt::aligned(plan, 128), "gpt_decode_fused_plan: plan must be 128-byte aligned");
  std::vector<uint8_t> host((size_t)gpt_decode_fused_plan_bytes(L), 0);
  CUtensorMap* maps = reinterpret_cast<CUtensorMap*>(host.data());
  LayerW* lw = reinterpret_cast<LayerW*>(host.data() + L * kPhases * sizeof(CUtensorMap));
  for (int64_t l = 0; l < L; ++l) {
    // per block: ln1_w, ln1_b, w_qkv, b_qkv, w_proj, b_proj, ln2_w, ln2_b, w_fc, b_fc, w_proj2, b_proj2
    const void* const* q = ptrs + l * 12;
    for (int i = 0; i < 12; ++i) GPT_CHECK_ARG(q[i] != nullptr, "gpt_decode_fused_plan: null weight %d of block %lld", i, (long long)l);
    for (int i : {2, 4, 8, 10})
      GPT_CHECK_ALIGN(gpt::aligned(q[i], 16), "gpt_decode_fused_plan: weights must be 16-byte aligned");
    const int64_t NK[4][2] = {{3 * C, C}, {C, C}, {4 * C, C}, {C, 4 * C}};
    const int widx[4] = {2, 4, 8, 10};
    for (int ph = 0; ph < kPhases; ++ph) {
      int s = gpt::tc::make_map(&maps[l * kPhases + ph], q[widx[ph]], NK[ph][0], NK[ph][1], NK[ph][1], 128);
      if (s) return s;
    }
    lw[l].ln1_w = (const __nv_bfloat16*)q[0];
    lw[l].ln1_b = (const __nv_bfloat16*)q[1];
    lw[l].b_qkv = (const __nv_bfloat16*)q[3];
    lw[l].b_proj = (const __nv_bfloat16*)q[5];
    lw[l].ln2_w = (const __nv_bfloat16*)q[6];
    lw[l].ln2_b = (const __nv_bfloat16*)q[7];
    lw[l].b_fc = (const __nv_bfloat16*)q[9];
    lw[l].b_proj2 = (const __nv_bfloat16*)q[11];
  }
  cudaError_t e = cudaMemcpy(plan, host.data(), host.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return gpt::fail(GPT_ERR_CUDA, "gpt_decode_fused_plan: %s", cudaGetErrorString(e));
  return GPT_OK;
}

int gpt_decode_fused(const void* plan, int64_t L, int64_t C, int64_t B, int64_t Tmax, const int64_t* tok,
                     const int64_t* pos_dev, const void* wte, int64_t vocab, const void* wpe, int64_t n_pos, const void* lnf_w,
                     const void* lnf_b, void* kv_cache, void* h_out, void* workspace, int64_t workspace_bytes,
                     void* stream) {
  using namespace gpt::fused;
  GPT_CHECK_SHAPE(L > 0 && C > 0 && C % 128 == 0 && C <= kCompute * kMaxPerThread && B > 0 && B <= kMaxMp && Tmax > 0 && n_pos > 0,
                  "gpt_decode_fused: unsupported sizes L=%lld C=%lld B=%lld", (long long)L, (long long)C, (long long)B);
  GPT_CHECK_ARG(plan && tok && pos_dev && wte && wpe && lnf_w && lnf_b && kv_cache && h_out && workspace,
                "gpt_decode_fused: null pointer");
  const int Mp = B <= 32 ? 32 : 64;
  GPT_CHECK_SHAPE(workspace_bytes >= ws_bytes(C, Mp), "gpt_decode_fused: workspace of %lld bytes required",
                  (long long)ws_bytes(C, Mp));
  GPT_CHECK_ALIGN(gpt::aligned(workspace, 256) && gpt::aligned(h_out, 16) && gpt::aligned(kv_cache, 16),
                  "gpt_decode_fused: workspace 256-byte, h_out / cache 16-byte aligned");
  const int sms = gpt::device_sm_count();
  if (sms <= 0) return gpt::fail(GPT_ERR_CUDA, "no CUDA device");
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(decode_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return gpt::fail(GPT_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    attr_done[dev] = true;
  }
  Params p;
  p.maps = reinterpret_cast<const CUtensorMap*>(plan);
  p.layers = reinterpret_cast<const LayerW*>((const uint8_t*)plan + L * kPhases * sizeof(CUtensorMap));
  p.L = (int)L;
  p.C = (int)C;
  p.H = (int)(C / 64);
  p.B = (int)B;
  p.Mp = Mp;
  p.Tmax = (int)Tmax;
  p.n_pos = (int)n_pos;
  p.vocab = (int)vocab;
  p.eps = 1e-5f;
  p.scale_log2 = (1.0f / 8.0f) * 1.4426950408889634f;   // 1/sqrt(64) * log2(e)
  p.tok = tok;
  p.pos_dev = pos_dev;
  p.wte = (const __nv_bfloat16*)wte;
  p.wpe = (const __nv_bfloat16*)wpe;
  p.lnf_w = (const __nv_bfloat16*)lnf_w;
  p.lnf_b = (const __nv_bfloat16*)lnf_b;
  p.cache = (__nv_bfloat16*)kv_cache;
  p.h_out = (__nv_bfloat16*)h_out;
  uint8_t* w = (uint8_t*)workspace;
  p.x = (__nv_bfloat16*)w;
  w += (int64_t)Mp * C * 2;
  p.att = (__nv_bfloat16*)w;
  w += (int64_t)Mp * C * 2;
  p.acc_qkv = (float*)w;
  w += 3 * C * (int64_t)Mp * 4;
  p.acc_proj = (float*)w;
  w += C * (int64_t)Mp * 4;
  p.acc_fc = (float*)w;
  w += 4 * C * (int64_t)Mp * 4;
  p.acc_fc2 = (float*)w;
  w += C * (int64_t)Mp * 4;
  p.stats = (float*)w;
  w += 4 * kMaxMp * 4;
  w = (uint8_t*)(((uintptr_t)w + 255) & ~(uintptr_t)255);
  p.bar = (unsigned long long*)w;
  // GPT_FUSED_TRACE=1: phase timestamps of CTA 0 go to the workspace tail (diagnostics).
  static const bool trace = [] {
    const char* e = getenv("GPT_FUSED_TRACE");
    return e && e[0] == '1';
  }();
  p.trace = trace ? (unsigned long long*)(w + 256) : nullptr;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;   // all CTAs co-resident: required by the grid barrier
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, decode_fused_kernel, p);
  if (e != cudaSuccess) return gpt::fail(GPT_ERR_CUDA, "gpt_decode_fused launch: %s", cudaGetErrorString(e));
  return gpt::launch_status("decode_fused");
}

}  // extern "C"
