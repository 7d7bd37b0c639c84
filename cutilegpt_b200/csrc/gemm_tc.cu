// bf16 dense contraction on the 5th-generation tensor cores (sm_100a):
//   C[M, N] = epilogue(A[M, K] · W[N, K]ᵀ)
// A is the activation (row stride lda), W the nn.Linear [out, in] weight.
// Both operands are K-major, which is the layout tcgen05.mma consumes
// directly, so no transposed weight copy exists (the reference keeps a
// second [in, out] copy of every weight, cutile_gpt/models/gpt.py:83-90).
//
// Structure (one persistent CTA per SM, 320 threads):
//   warp 0      TMA producer: A/W k-blocks (128 B rows, 128 B swizzle)
//               into a kStages-deep shared-memory ring, mbarrier tx counts.
//   warp 1      allocates TMEM; lane 0 issues tcgen05.mma (M=128, N=BN,
//               K=16 per instruction, fp32 accumulators in TMEM) and
//               tcgen05.commit to release ring slots / publish tiles.
//   warps 2-9   epilogue: tcgen05.ld 32 columns at a time, transpose
//               through shared memory so each warp store covers a
//               contiguous row segment, apply bias / GELU / residual,
//               convert, store. Two TMEM accumulators (2 × BN columns) let
//               the epilogue of tile i overlap the MMAs of tile i+1.
// Every mbarrier wait is bounded (kWaitLimitNs); on expiry the kernel
// records GPT_DEVERR_TIMEOUT and unwinds instead of spinning forever.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <stdlib.h>

#include "common.cuh"

namespace gpt {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one 128B-swizzle row
constexpr int kEpiWarps = 8;                       // epilogue warps, TMA-store variants
constexpr int kThreads = (2 + kEpiWarps) * 32;
// Epilogue warps of the LSU-store variant (row pitch not 16-byte aligned: the
// lm_head's 50257). With 16-byte chunk stores 8 warps and the deeper operand
// ring they leave room for beat 16 warps (1146 vs 1167 us at M=16384).
constexpr int epi_warps(bool tma_store) { return tma_store ? kEpiWarps : 8; }
constexpr int kStageRowPitch = 33;  // fp32 words per staged row (bank-conflict free)

struct Params {
  int M, N, K;
  int num_m, num_n, num_tiles, num_kb;
  int n_fast;  // tile order: 1 = the N tiles of one row block run together
  const __nv_bfloat16* bias;
  const __nv_bfloat16* resid;
  __nv_bfloat16* C;
  int64_t ldr, ldc;
  // FUSE = 1: LayerNorm folded in (A = raw rows x, W = gamma-scaled weight):
  //   C = rstd * (acc - mean * ln_u) + ln_v, mean / rstd from ln_stats [ln_parts][M][2]
  // FUSE = 2: per 128-column part, (sum, sum of squares) of the stored rows -> stats_out [ceil(N/128)][M][2]
  const float* ln_stats;
  const float* ln_u;
  const float* ln_v;
  int ln_parts;
  float ln_eps, ln_inv_k;
  float* stats_out;
};

// mean and rstd of row `row` from the per-part (sum, sum of squares) statistics.
__device__ __forceinline__ void ln_row_stats(const Params& p, int row, float& mean, float& rstd) {
  float s1 = 0.f, s2 = 0.f;
  for (int q = 0; q < p.ln_parts; ++q) {
    const float2 v = *reinterpret_cast<const float2*>(p.ln_stats + ((int64_t)q * p.M + row) * 2);
    s1 += v.x;
    s2 += v.y;
  }
  mean = s1 * p.ln_inv_k;
  rstd = rsqrtf(fmaxf(s2 * p.ln_inv_k - mean * mean, 0.f) + p.ln_eps);
}

// ---- PTX wrappers -----------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity to complete.
__device__ __noinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try(bar, parity)) return true;
    if (global_timer_ns() - t0 > g_wait_limit_ns) {
      record_device_error(GPT_DEVERR_TIMEOUT);
      return false;
    }
  }
}
// First try inline (the phase has usually completed already), the bounded spin out of line.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  return mbar_try(bar, parity) || mbar_wait_spin(bar, parity);
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// 32 consecutive bf16 values starting at p (16-byte aligned) -> floats.
__device__ __forceinline__ void load32_bf16(const __nv_bfloat16* p, float* out) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 raw = *reinterpret_cast<const uint4*>(p + 8 * i);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) out[8 * i + j] = __bfloat162float(e[j]);
  }
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accum) {
  uint32_t mask0 = 0, mask1 = 0, mask2 = 0, mask3 = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(mask0), "r"(mask1), "r"(mask2), "r"(mask3));
}
// 32 lanes x 32 consecutive fp32 columns: thread t of the warp receives
// row (quadrant*32 + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, K-major operand with 128-byte swizzle:
// rows of 128 B, 8-row swizzle atoms 1024 B apart (stride byte offset),
// descriptor version 1 (bits 46-47), layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
  d |= (uint64_t)1 << 46;             // version
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: D fp32, A/B bf16, both K-major.
template <int N_>
__device__ __forceinline__ constexpr uint32_t idesc_bf16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N_ >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// Pair mode (kPair): a 2-CTA cluster computes one 256 x BN tile with
// tcgen05.mma.cta_group::2 (M = 256). Each CTA loads its own 128 A rows and
// half of the BN W rows, so a CTA streams 128 x 64 + BN/2 x 64 operand
// elements per k-block instead of 128 x 64 + BN x 64: a third less L2 ->
// shared-memory traffic per FLOP. The even CTA (leader) issues the MMAs;
// each CTA's TMEM holds the accumulators of its own 128 rows, which its own
// epilogue warps drain. All loads are plain per-CTA TMA loads (no multicast);
// only the MMA completion (tcgen05.commit) is multicast to both CTAs.
template <int BN, bool kPair, int kEW = kEpiWarps>
struct Smem {
  static constexpr int kBRows = kPair ? BN / 2 : BN;
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = kBRows * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // ring depth: what fits beside the epilogue staging (kEW warps x 4.2 KB)
  static constexpr int kStages = kEW > kEpiWarps ? (kStageBytes <= 32768 ? 4 : 3)
                                                 : (kPair ? 6 : (BN >= 256 ? 4 : 6));
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kEpiBytes = kEW * 32 * kStageRowPitch * 4;
  static constexpr int kBarBytes = (2 * kStages + 4) * 8 + 16;
  static constexpr int kTotal = 1024 + kRingBytes + kEpiBytes + kBarBytes;
  static constexpr int kTmemCols = 2 * BN;  // double-buffered accumulator
};

__device__ __forceinline__ uint32_t cta_rank_in_cluster() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same shared-memory location in CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(local), "r"(rank));
  return out;
}
// Pair-mode TMA load: the bytes land in this CTA's shared memory and are
// counted on `bar`, which may be the leader CTA's barrier (cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accum) {
  const uint32_t z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n}\n" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(z));
}
// Arrive on the barrier at this shared-memory offset in both CTAs of the
// pair once every previously issued MMA of this thread has completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          bar),
      "h"((uint16_t)0x3)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// Accumulator release by an epilogue warp: what the MMA issuer must not
// overtake is this warp's TMEM reads, which tcgen05.wait::ld completed and
// tcgen05.fence::before_thread_sync ordered. No memory needs releasing, so the
// arrive is relaxed: a release at cluster scope would first wait for every
// global store the warp has in flight.
__device__ __forceinline__ void mbar_arrive_tmem_free(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

template <int BN, int EPI, bool kTmaStore, bool kPair, int FUSE = 0>
__global__ void __launch_bounds__((2 + epi_warps(kTmaStore)) * 32, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const Params p) {
  constexpr int kEW = epi_warps(kTmaStore);
  using S = Smem<BN, kPair, kEW>;
  constexpr int kStages = S::kStages;
  constexpr int kTileM = kPair ? 2 * BM : BM;
  extern __shared__ uint8_t smem_dyn[];
  // 1024-byte alignment is required by the 128B swizzle atoms.
  uint8_t* base = (uint8_t*)(((uintptr_t)smem_dyn + 1023) & ~(uintptr_t)1023);
  uint8_t* ringA = base;
  uint8_t* ringB = base + kStages * S::kABytes;
  float* epi = (float*)(base + S::kRingBytes);
  uint64_t* bars = (uint64_t*)(base + S::kRingBytes + S::kEpiBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* tfull = bars + 2 * kStages;
  uint64_t* tempty = bars + 2 * kStages + 2;
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * kStages + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = kPair ? cta_rank_in_cluster() : 0u;  // 0 = leader
  const int first_tile = kPair ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tile_step = kPair ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_addr(&tfull[a]), 1);
      // Pair mode: the leader's accumulator is free once the epilogue warps
      // of both CTAs have drained it.
      mbar_init(smem_addr(&tempty[a]), kPair ? 2 * kEW : kEW);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 1) {
    if constexpr (kPair) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_addr(tmem_slot)),
                   "r"((uint32_t)S::kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_addr(tmem_slot)),
                   "r"((uint32_t)S::kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (kPair) cluster_barrier();  // peer barriers initialised before any remote arrive / TMA
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above touched only this CTA's (pair's) resources; from here on
  // the kernel reads activations and writes outputs of the stream.
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = first_tile; tile < p.num_tiles && ok; tile += tile_step) {
        const int m_blk = p.n_fast ? tile / p.num_n : tile % p.num_m;
        const int n_blk = p.n_fast ? tile % p.num_n : tile / p.num_m;
        const int a_row = m_blk * kTileM + (int)rank * BM;
        const int b_row = n_blk * BN + (int)rank * S::kBRows;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(smem_addr(&empty[stage]), phase ^ 1)) { ok = false; break; }
          if constexpr (kPair) {
            // Both CTAs' bytes are counted on the leader's barrier.
            const uint32_t fb = cluster_addr(smem_addr(&full[stage]), 0);
            if (rank == 0) mbar_expect_tx(smem_addr(&full[stage]), 2 * S::kStageBytes);
            tma_load_2d_pair(smem_addr(ringA + stage * S::kABytes), &tmA, fb, kb * BK, a_row);
            tma_load_2d_pair(smem_addr(ringB + stage * S::kBBytes), &tmB, fb, kb * BK, b_row);
          } else {
            const uint32_t fb = smem_addr(&full[stage]);
            mbar_expect_tx(fb, S::kStageBytes);
            tma_load_2d(smem_addr(ringA + stage * S::kABytes), &tmA, fb, kb * BK, a_row);
            tma_load_2d(smem_addr(ringB + stage * S::kBBytes), &tmB, fb, kb * BK, b_row);
          }
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                 ((uint32_t)(kTileM >> 4) << 24);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const uint64_t ad0 = desc_sw128(smem_addr(ringA)), bd0 = desc_sw128(smem_addr(ringB));
      for (int tile = first_tile; tile < p.num_tiles && ok; tile += tile_step) {
        if (!mbar_wait(smem_addr(&tempty[acc]), acc_phase ^ 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(smem_addr(&full[stage]), phase)) { ok = false; break; }
          tc_fence_after();
          // descriptors of this stage: the address field (bytes >> 4) offset from stage 0
          const uint64_t ad = ad0 + (uint64_t)(stage * (S::kABytes >> 4));
          const uint64_t bd = bd0 + (uint64_t)(stage * (S::kBBytes >> 4));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // +32 bytes per K=16 step inside the swizzle atom (encoded >>4).
            if constexpr (kPair)
              tc_mma_pair(d_tmem, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (kb | k) != 0);
            else
              tc_mma(d_tmem, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (kb | k) != 0);
          }
          // slot free (in both CTAs) once these MMAs retire
          if constexpr (kPair) tc_commit_pair(smem_addr(&empty[stage]));
          else tc_commit(smem_addr(&empty[stage]));
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        // accumulator ready for the epilogue(s)
        if constexpr (kPair) tc_commit_pair(smem_addr(&tfull[acc]));
        else tc_commit(smem_addr(&tfull[acc]));
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  } else {
    const uint32_t tempty_leader[2] = {kPair ? cluster_addr(smem_addr(&tempty[0]), 0) : smem_addr(&tempty[0]),
                                       kPair ? cluster_addr(smem_addr(&tempty[1]), 0) : smem_addr(&tempty[1])};
    if constexpr (kTmaStore) {
      // ---------------------------------------------------------- epilogue (TMA store)
      // lane == row: 32 accumulator columns from TMEM, bias / GELU / residual in
      // registers, packed bf16 into a 32x32 staging tile (64B-swizzled rows),
      // written by one TMA bulk store per chunk. Two staging tiles per warp so
      // the next chunk's math overlaps the previous store.
      const int ew = warp - 2;
      const int quad = warp & 3;
      const int half = ew >> 2;
      uint8_t* stg = reinterpret_cast<uint8_t*>(epi) + ew * 4096;
      constexpr int kChunksPerHalf = BN / 64;
      int sb = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = first_tile; tile < p.num_tiles; tile += tile_step) {
        const int m_blk = p.n_fast ? tile / p.num_n : tile % p.num_m;
        const int n_blk = p.n_fast ? tile % p.num_n : tile / p.num_m;
        const int row0 = m_blk * kTileM + (int)rank * BM + quad * 32;
        const int row = row0 + lane;
        const bool row_ok = row < p.M;
        float ln_mean = 0.f, ln_rstd = 1.f;
        if (FUSE == 1 && row_ok) ln_row_stats(p, row, ln_mean, ln_rstd);
        float st1 = 0.f, st2 = 0.f;   // FUSE == 2: this row's sums over the warp's columns
        // The residual row segments of every chunk of this tile are requested
        // before waiting for the accumulator, so their HBM latency overlaps
        // the tile's MMAs instead of serialising chunk after chunk.
        uint4 rraw[kChunksPerHalf][4];
        if (EPI == GPT_EPI_BIAS_RESIDUAL) {
#pragma unroll
          for (int cc = 0; cc < kChunksPerHalf; ++cc) {
            const int col0 = n_blk * BN + (half * kChunksPerHalf + cc) * 32;
            if (row_ok && col0 + 32 <= p.N) {
              const uint4* rp = reinterpret_cast<const uint4*>(p.resid + (int64_t)row * p.ldr + col0);
#pragma unroll
              for (int i = 0; i < 4; ++i) rraw[cc][i] = __ldg(rp + i);
            }
          }
        }
        if (!mbar_wait(smem_addr(&tfull[acc]), acc_phase)) break;
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < kChunksPerHalf; ++cc) {
          const int c = half * kChunksPerHalf + cc;
          const int col0 = n_blk * BN + c * 32;
          const bool full = col0 + 32 <= p.N;
          // bias and residual stay packed (bf16 pairs) until the math loop
          // (with the LayerNorm fold the bias is part of ln_v and may be null).
          uint32_t bw[16], rw[16];
          if (EPI != GPT_EPI_NONE && FUSE != 1) {
            if (full) {
              const uint4* bp = reinterpret_cast<const uint4*>(p.bias + col0);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint4 v = __ldg(bp + i);
                bw[4 * i] = v.x; bw[4 * i + 1] = v.y; bw[4 * i + 2] = v.z; bw[4 * i + 3] = v.w;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float lo = col0 + 2 * j < p.N ? __bfloat162float(p.bias[col0 + 2 * j]) : 0.f;
                const float hi = col0 + 2 * j + 1 < p.N ? __bfloat162float(p.bias[col0 + 2 * j + 1]) : 0.f;
                bw[j] = pack2_bf16(lo, hi);
              }
            }
          }
          if (EPI == GPT_EPI_BIAS_RESIDUAL) {
            if (row_ok && full) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                rw[4 * i] = rraw[cc][i].x; rw[4 * i + 1] = rraw[cc][i].y;
                rw[4 * i + 2] = rraw[cc][i].z; rw[4 * i + 3] = rraw[cc][i].w;
              }
            } else {
              const __nv_bfloat16* rp = p.resid + (int64_t)row * p.ldr + col0;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float lo = (row_ok && col0 + 2 * j < p.N) ? __bfloat162float(rp[2 * j]) : 0.f;
                const float hi = (row_ok && col0 + 2 * j + 1 < p.N) ? __bfloat162float(rp[2 * j + 1]) : 0.f;
                rw[j] = pack2_bf16(lo, hi);
              }
            }
          }
          uint32_t r[32];
          tmem_ld32(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float v0 = __uint_as_float(r[2 * j]), v1 = __uint_as_float(r[2 * j + 1]);
            if (FUSE == 1) {
              // LayerNorm fold; u / v of these two columns (the same for every row: L1 hits)
              const int cc0 = col0 + 2 * j;
              const float2 uu = full ? __ldg(reinterpret_cast<const float2*>(p.ln_u + cc0))
                                     : make_float2(cc0 < p.N ? p.ln_u[cc0] : 0.f, cc0 + 1 < p.N ? p.ln_u[cc0 + 1] : 0.f);
              const float2 vv = full ? __ldg(reinterpret_cast<const float2*>(p.ln_v + cc0))
                                     : make_float2(cc0 < p.N ? p.ln_v[cc0] : 0.f, cc0 + 1 < p.N ? p.ln_v[cc0 + 1] : 0.f);
              v0 = ln_rstd * (v0 - ln_mean * uu.x) + vv.x;
              v1 = ln_rstd * (v1 - ln_mean * uu.y) + vv.y;
            } else if (EPI != GPT_EPI_NONE) {
              const float2 bf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bw[j]));
              v0 += bf.x; v1 += bf.y;
            }
            if (EPI == GPT_EPI_BIAS_GELU) gelu_tanh2_fast(v0, v1);
            if (EPI == GPT_EPI_BIAS_RESIDUAL) {
              const float2 rf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rw[j]));
              v0 += rf.x; v1 += rf.y;
            }
            pk[j] = pack2_bf16(v0, v1);
            if (FUSE == 2) {   // statistics of the stored (rounded) values; columns past N hold 0
              const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&pk[j]));
              st1 += y.x + y.y;
              st2 = fmaf(y.x, y.x, fmaf(y.y, y.y, st2));
            }
          }
          // The store issued from this staging tile two chunks ago must have read it.
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          __syncwarp();
          uint8_t* tile_s = stg + sb * 2048;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int phys = k ^ ((lane >> 1) & 3);  // 64-byte swizzle of the tensor map
            *reinterpret_cast<uint4*>(tile_s + lane * 64 + phys * 16) =
                make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, smem_addr(tile_s), col0, row0);
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          sb ^= 1;
        }
        if (FUSE == 2 && row_ok) {   // part = 128-column half of the BN = 256 tile
          *reinterpret_cast<float2*>(p.stats_out + ((int64_t)(n_blk * 2 + half) * p.M + row) * 2) =
              make_float2(st1, st2);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (kPair) mbar_arrive_tmem_free(tempty_leader[acc]);
          else mbar_arrive(tempty_leader[acc]);
        }
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    } else {
      // ---------------------------------------------------------- epilogue (LSU stores)
      // Any row pitch (the lm_head output has an odd one): lane == row to stage
      // the accumulators in shared memory, then lane == column for coalesced
      // stores of each row segment.
      const int ew = warp - 2;             // 0 .. kEW-1
      const int quad = warp & 3;           // TMEM lane quadrant this warp may access
      const int half = ew >> 2;            // which part (of kEW / 4) of the BN columns
      float* stg = epi + ew * 32 * kStageRowPitch;
      constexpr int kChunks = BN / 32;
      constexpr int kChunksPerHalf = kChunks / (kEW / 4);
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = first_tile; tile < p.num_tiles; tile += tile_step) {
        const int m_blk = p.n_fast ? tile / p.num_n : tile % p.num_m;
        const int n_blk = p.n_fast ? tile % p.num_n : tile / p.num_m;
        if (!mbar_wait(smem_addr(&tfull[acc]), acc_phase)) break;
        tc_fence_after();
        const int row0 = m_blk * kTileM + (int)rank * BM + quad * 32;
        float ln_mean = 0.f, ln_rstd = 1.f;   // FUSE == 1: statistics of row row0 + lane
        if (FUSE == 1 && row0 + lane < p.M) ln_row_stats(p, row0 + lane, ln_mean, ln_rstd);
        if constexpr (EPI == GPT_EPI_NONE) {
          // No bias / residual (the lm_head): lane == row finishes its values and
          // stages them as packed bf16; then each row segment is written as the
          // 16-byte-aligned chunks it contains (8 bf16 per st.global.v4, shifted
          // by one element when the row starts on an odd element) plus its few
          // edge elements. A row of the odd 50257 pitch starts at element
          // offset row mod 8 inside a 16-byte unit.
          // A warp's columns go in passes of at most 64 (32 packed words per
          // staged row, inside the 33-word pitch).
          constexpr int kSub = kChunksPerHalf < 2 ? kChunksPerHalf : 2;   // 32-column chunks per pass
          constexpr int kSeg = kSub * 32;             // columns of one pass
          constexpr int kLpr = kSeg / 8;              // lanes per row (one 16-byte chunk each)
          constexpr int kRpi = 32 / kLpr;             // rows per store iteration
          static_assert(kSeg / 2 <= kStageRowPitch, "staged row exceeds the pitch");
          uint32_t* sw = reinterpret_cast<uint32_t*>(stg);   // 32 rows x 33 words
#pragma unroll 1
          for (int pass = 0; pass < kChunksPerHalf / kSub; ++pass) {
          const int chunk0 = half * kChunksPerHalf + pass * kSub;
          const int colseg = n_blk * BN + chunk0 * 32;
#pragma unroll
          for (int cc = 0; cc < kSub; ++cc) {
            uint32_t r[32];
            tmem_ld32(tmem_base + ((uint32_t)(quad * 32) << 16) +
                          (uint32_t)(acc * BN + (chunk0 + cc) * 32), r);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float v0 = __uint_as_float(r[2 * j]), v1 = __uint_as_float(r[2 * j + 1]);
              if (FUSE == 1) {
                const int c0 = colseg + cc * 32 + 2 * j;
                const float u0 = c0 < p.N ? p.ln_u[c0] : 0.f, u1 = c0 + 1 < p.N ? p.ln_u[c0 + 1] : 0.f;
                const float w0 = c0 < p.N ? p.ln_v[c0] : 0.f, w1 = c0 + 1 < p.N ? p.ln_v[c0 + 1] : 0.f;
                v0 = ln_rstd * (v0 - ln_mean * u0) + w0;
                v1 = ln_rstd * (v1 - ln_mean * u1) + w1;
              }
              sw[lane * kStageRowPitch + cc * 16 + j] = pack2_bf16(v0, v1);
            }
          }
          __syncwarp();
          const int k8 = lane % kLpr, rsub = lane / kLpr;
          uint16_t* C16 = reinterpret_cast<uint16_t*>(p.C);
          const int c_mis = (int)((reinterpret_cast<uintptr_t>(p.C) >> 1) & 7);
          if (colseg + kSeg <= p.N) {
#pragma unroll
            for (int rr0 = 0; rr0 < 32; rr0 += kRpi) {
              const int rr = rr0 + rsub;
              const int row = row0 + rr;
              if (row < p.M) {
                const int64_t g0 = (int64_t)row * p.ldc + colseg;   // element index of the segment
                const int head = (8 - (int)((c_mis + g0) & 7)) & 7;  // elements before the first 16-byte boundary
                const int nfull = (kSeg - head) >> 3;
                const uint32_t* srow = sw + rr * kStageRowPitch;
                if (k8 < nfull) {
                  const int e0 = head + 8 * k8;
                  const int b = e0 >> 1;
                  uint32_t w[4];
                  if ((e0 & 1) == 0) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) w[i] = srow[b + i];
                  } else {
                    uint32_t t[5];
#pragma unroll
                    for (int i = 0; i < 5; ++i) t[i] = srow[b + i];
#pragma unroll
                    for (int i = 0; i < 4; ++i) w[i] = __funnelshift_r(t[i], t[i + 1], 16);
                  }
                  asm volatile("st.global.cs.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(C16 + g0 + e0), "r"(w[0]),
                               "r"(w[1]), "r"(w[2]), "r"(w[3])
                               : "memory");
                }
                // the (head + tail) = 8 edge elements when the segment is not aligned
                if (head != 0) {
                  for (int i = k8; i < 8; i += kLpr) {
                    const int e = i < head ? i : kSeg - 8 + i;
                    C16[g0 + e] = (uint16_t)(srow[e >> 1] >> ((e & 1) * 16));
                  }
                }
              }
            }
          } else {
            // the segment crosses N (last vocabulary tile): element stores, lane == column
#pragma unroll 1
            for (int rr = 0; rr < 32; ++rr) {
              const int row = row0 + rr;
              if (row >= p.M) break;
              for (int e = lane; e < kSeg; e += 32)
                if (colseg + e < p.N)
                  C16[(int64_t)row * p.ldc + colseg + e] =
                      (uint16_t)(sw[rr * kStageRowPitch + (e >> 1)] >> ((e & 1) * 16));
            }
          }
          __syncwarp();
          }  // pass
        } else
        for (int c = half * kChunksPerHalf; c < (half + 1) * kChunksPerHalf; ++c) {
          // lane == column in the store phase below.
          const int col = n_blk * BN + c * 32 + lane;
          const bool col_ok = col < p.N;
          // Residual loads for all 32 rows are issued first so their latency
          // overlaps the TMEM load and the shared-memory transpose.
          float res[32];
          if (EPI == GPT_EPI_BIAS_RESIDUAL) {
#pragma unroll
            for (int rr = 0; rr < 32; ++rr) {
              const int row = row0 + rr;
              res[rr] = (row < p.M && col_ok) ? __bfloat162float(p.resid[(int64_t)row * p.ldr + col]) : 0.f;
            }
          }
          float bcol = 0.f, ucol = 0.f;
          if (FUSE == 1) {
            if (col_ok) {
              ucol = p.ln_u[col];
              bcol = p.ln_v[col];
            }
          } else if (EPI != GPT_EPI_NONE && col_ok) {
            bcol = __bfloat162float(p.bias[col]);
          }
          uint32_t r[32];
          const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN + c * 32);
          tmem_ld32(taddr, r);
          // lane == row: stage the raw accumulators.
#pragma unroll
          for (int j = 0; j < 32; ++j) stg[lane * kStageRowPitch + j] = __uint_as_float(r[j]);
          __syncwarp();
          // lane == column: bias / GELU / residual, coalesced row stores.
#pragma unroll
          for (int rr = 0; rr < 32; ++rr) {
            const int row = row0 + rr;
            const float mrr = FUSE == 1 ? __shfl_sync(0xffffffffu, ln_mean, rr) : 0.f;
            const float rrr = FUSE == 1 ? __shfl_sync(0xffffffffu, ln_rstd, rr) : 1.f;
            if (row < p.M && col_ok) {
              float v = stg[rr * kStageRowPitch + lane];
              v = FUSE == 1 ? rrr * (v - mrr * ucol) + bcol : v + bcol;
              if (EPI == GPT_EPI_BIAS_GELU) v = gelu_tanh<true>(v);
              if (EPI == GPT_EPI_BIAS_RESIDUAL) v += res[rr];
              p.C[(int64_t)row * p.ldc + col] = __float2bfloat16_rn(v);
            }
          }
          __syncwarp();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (kPair) mbar_arrive_tmem_free(tempty_leader[acc]);
          else mbar_arrive(tempty_leader[acc]);
        }
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // Pair mode: neither CTA frees its TMEM or shared memory while the peer may
  // still issue MMAs into it or arrive on its barriers.
  if constexpr (kPair) cluster_barrier();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (kPair)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"((uint32_t)S::kTmemCols));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"((uint32_t)S::kTmemCols));
  }
}

// ---- host side ---------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)ptr;
    else
      cudaGetLastError();
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with row pitch
// `ld` elements; box = box_rows x 64 columns, 128-byte swizzle, OOB -> 0.
static int make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld,
                    int box_rows, int box_cols = BK,
                    CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto enc = get_encode();
  if (!enc) return fail(GPT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GPT_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return GPT_OK;
}

template <int BN, int EPI, bool kTmaStore, bool kPair, int FUSE = 0>
static int launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tcm, const Params& p,
                     int grid, cudaStream_t st) {
  constexpr int kEW = epi_warps(kTmaStore);
  constexpr int kThr = (2 + kEW) * 32;
  using S = Smem<BN, kPair, kEW>;
  static_assert(S::kTotal <= 232448, "shared memory budget exceeded");
  static_assert(S::kEpiBytes >= kEpiWarps * 4096, "TMA-store staging does not fit");
  auto kern = gemm_tc_kernel<BN, EPI, kTmaStore, kPair, FUSE>;
  // Attribute set per device the first time this instantiation runs there.
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> g(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
      if (e != cudaSuccess) return fail(GPT_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      done[dev] = true;
    }
  }
  if constexpr (kPair)
    launch_pdl_cluster(kern, dim3(grid), dim3(kThr), S::kTotal, st, 2u, ta, tb, tcm, p);
  else
    launch_pdl(kern, dim3(grid), dim3(kThr), S::kTotal, st, ta, tb, tcm, p);
  return launch_status("gemm_tc");
}

// Tile width: 256 unless N is at most 128. Measured on B200 at M = 16384
// (K = 768 / 3072): BN = 256 is faster for every GPT-2 GEMM, even where the
// 128-wide tile quantises better over 148 SMs (c_fc + GELU: 77 us vs 118 us).
// A 256 x 128 CTA-pair tile was slower still for every shape (attn c_proj,
// N = K = 768: 41.8 us vs 34.8 us; QKV 86.8 vs 54.1 us).
static int pick_bn(int64_t M, int64_t N, int sms) {
  (void)M;
  (void)sms;
  return N <= 128 ? 128 : 256;
}

// Co-resident 2-CTA clusters of the pair kernel on this device (the GPC
// layout can leave SMs without a partner); the persistent grid never exceeds it.
static int pair_slots(int sms) {
  static int cached[64] = {0};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return sms / 2;
  std::lock_guard<std::mutex> g(mu);
  if (cached[dev] == 0) {
    using S = Smem<256, true>;
    auto kern = gemm_tc_kernel<256, GPT_EPI_NONE, true, true>;
    int n = sms / 2;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * n);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = S::kTotal;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) == cudaSuccess && clusters > 0 && clusters < n)
        n = clusters;
    }
    cudaGetLastError();
    cached[dev] = n;
  }
  return cached[dev];
}

template <int BN, bool kPair>
static int launch_epi(int epi, bool tma_store, const CUtensorMap& ta, const CUtensorMap& tb,
                      const CUtensorMap& tcm, const Params& p, int grid, cudaStream_t st) {
#define GPT_TC_EPI(TS)                                                                                     \
  switch (epi) {                                                                                           \
    case GPT_EPI_NONE: return launch_bn<BN, GPT_EPI_NONE, TS, kPair>(ta, tb, tcm, p, grid, st);           \
    case GPT_EPI_BIAS: return launch_bn<BN, GPT_EPI_BIAS, TS, kPair>(ta, tb, tcm, p, grid, st);           \
    case GPT_EPI_BIAS_GELU: return launch_bn<BN, GPT_EPI_BIAS_GELU, TS, kPair>(ta, tb, tcm, p, grid, st); \
    default: return launch_bn<BN, GPT_EPI_BIAS_RESIDUAL, TS, kPair>(ta, tb, tcm, p, grid, st);            \
  }
  if (tma_store) { GPT_TC_EPI(true) } else { GPT_TC_EPI(false) }
#undef GPT_TC_EPI
}

int gemm_bf16(const void* A, int64_t lda, const void* W, const void* bias, const void* R, int64_t ldr,
              void* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int epi, cudaStream_t st,
              const gpt_gemm_fusion* fusion) {
  const bool f_ln = fusion && fusion->ln_stats;
  const bool f_st = fusion && fusion->row_stats;
  int sms = device_sm_count();
  if (sms <= 0) return fail(GPT_ERR_CUDA, "no CUDA device");
  int bn = pick_bn(M, N, sms);
  // CTA pairs (256-row tiles, cta_group::2) for BN = 256 once there are
  // enough rows to fill them.
  const bool pair = bn == 256 && sms >= 2 && M > BM;
  const int tile_m = pair ? 2 * BM : BM;
  CUtensorMap ta, tb;
  int s = make_map(&ta, A, M, K, lda, BM);
  if (s) return s;
  s = make_map(&tb, W, N, K, K, pair ? bn / 2 : bn);
  if (s) return s;
  Params p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.num_m = (int)((M + tile_m - 1) / tile_m);
  p.num_n = (int)((N + bn - 1) / bn);
  p.num_tiles = p.num_m * p.num_n;
  p.num_kb = (int)((K + BK - 1) / BK);
  // Row blocks of A are read from HBM once either way; the order decides
  // which operand is re-read from L2. N-fastest keeps one row block of A hot
  // while every N tile consumes it, which needs all of W resident in L2:
  // chosen while W is small (every GPT-2 layer weight), otherwise M-fastest
  // (the 77 MB lm_head weight is then streamed once, A re-read from L2).
  p.n_fast = (N * K * 2 <= (32ll << 20)) ? 1 : 0;
  p.bias = (const __nv_bfloat16*)bias;
  p.resid = (const __nv_bfloat16*)R;
  p.C = (__nv_bfloat16*)C;
  p.ldr = ldr;
  p.ldc = ldc;
  p.ln_stats = f_ln ? fusion->ln_stats : nullptr;
  p.ln_u = f_ln ? fusion->ln_u : nullptr;
  p.ln_v = f_ln ? fusion->ln_v : nullptr;
  p.ln_parts = f_ln ? (int)fusion->ln_parts : 0;
  p.ln_eps = f_ln ? fusion->ln_eps : 0.f;
  p.ln_inv_k = 1.0f / (float)K;
  p.stats_out = f_st ? fusion->row_stats : nullptr;
  const int slots = pair ? pair_slots(sms) : sms;  // persistent CTAs (pairs)
  int grid = p.num_tiles < slots ? p.num_tiles : slots;
  if (pair) grid *= 2;
  // TMA-store epilogue when C (and R) rows are 16-byte aligned; otherwise LSU stores.
  const bool tma_store = aligned(C, 16) && (ldc * 2) % 16 == 0 &&
                         (epi != GPT_EPI_BIAS_RESIDUAL || (aligned(R, 16) && (ldr * 2) % 16 == 0)) &&
                         (epi == GPT_EPI_NONE || f_ln || aligned(bias, 16));
  CUtensorMap tcm;
  if (tma_store) {
    s = make_map(&tcm, C, M, N, ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    if (s) return s;
  } else {
    tcm = ta;  // unused by the LSU-store epilogue
  }
  if (f_ln || f_st) {
    // Fused prefill variants: CTA-pair tiles of 256 columns (row statistics are
    // kept per 128-column half tile); LayerNorm fold with none / bias / GELU,
    // row statistics with the residual epilogue (TMA-store path).
    if (!pair || bn != 256) return fail(GPT_ERR_UNSUPPORTED, "fused tcgen05 GEMM needs 256-wide CTA-pair tiles");
    if (f_ln && f_st) return fail(GPT_ERR_UNSUPPORTED, "LayerNorm fold and row statistics in one GEMM");
    if (f_st) {
      if (epi != GPT_EPI_BIAS_RESIDUAL || !tma_store)
        return fail(GPT_ERR_UNSUPPORTED, "row statistics need the aligned bias + residual epilogue");
      return launch_bn<256, GPT_EPI_BIAS_RESIDUAL, true, true, 2>(ta, tb, tcm, p, grid, st);
    }
    switch (epi) {
      case GPT_EPI_NONE:
        return tma_store ? launch_bn<256, GPT_EPI_NONE, true, true, 1>(ta, tb, tcm, p, grid, st)
                         : launch_bn<256, GPT_EPI_NONE, false, true, 1>(ta, tb, tcm, p, grid, st);
      case GPT_EPI_BIAS:
        if (!tma_store) return fail(GPT_ERR_UNSUPPORTED, "LayerNorm fold with bias needs an aligned output");
        return launch_bn<256, GPT_EPI_BIAS, true, true, 1>(ta, tb, tcm, p, grid, st);
      case GPT_EPI_BIAS_GELU:
        if (!tma_store) return fail(GPT_ERR_UNSUPPORTED, "LayerNorm fold with GELU needs an aligned output");
        return launch_bn<256, GPT_EPI_BIAS_GELU, true, true, 1>(ta, tb, tcm, p, grid, st);
      default:
        return fail(GPT_ERR_UNSUPPORTED, "LayerNorm fold with a residual epilogue");
    }
  }
  if (bn == 256) {
    if (pair) return launch_epi<256, true>(epi, tma_store, ta, tb, tcm, p, grid, st);
    return launch_epi<256, false>(epi, tma_store, ta, tb, tcm, p, grid, st);
  }
  return launch_epi<128, false>(epi, tma_store, ta, tb, tcm, p, grid, st);
}

// Whether the tensor-core path can serve this request (TMA: 16-byte
// aligned base addresses and row pitches).
bool tc_eligible(const void* A, int64_t lda, const void* W, int64_t K, int64_t M, int64_t N) {
  return aligned(A, 16) && aligned(W, 16) && (lda * 2) % 16 == 0 && (K * 2) % 16 == 0 && K > 0 &&
         M > 0 && N > 0 && M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31);
}

}  // namespace tc
}  // namespace gpt

namespace gpt {
namespace tc {

// Self-test of the bounded wait: one CTA initialises an mbarrier that
// expects `expected` arrivals, makes `arrivals` of them and waits for the
// phase with the library's bounded wait (mbar_wait). With fewer arrivals
// than expected the wait runs out after the current limit and records
// GPT_DEVERR_TIMEOUT; out[0] = 1 if the phase completed, 0 if it timed out.
__global__ void selftest_wait_kernel(int expected, int arrivals, int* out) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_addr(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, (uint32_t)expected);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if ((int)threadIdx.x < arrivals) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(b) : "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) out[0] = mbar_wait(b, 0) ? 1 : 0;
}

}  // namespace tc
}  // namespace gpt

extern "C" int gpt_selftest_wait(int expected, int arrivals, int* out_dev, void* stream) {
  GPT_CHECK_ARG(out_dev != nullptr, "gpt_selftest_wait: null out_dev");
  GPT_CHECK_SHAPE(expected >= 1 && expected <= 32 && arrivals >= 0 && arrivals <= expected,
                  "gpt_selftest_wait: needs 1 <= expected <= 32 and 0 <= arrivals <= expected");
  gpt::tc::selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(expected, arrivals, out_dev);
  return gpt::launch_status("selftest_wait");
}
