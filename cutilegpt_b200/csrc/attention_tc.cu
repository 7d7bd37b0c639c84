// Causal prefill attention on the 5th-generation tensor cores (bf16,
// head_dim 64), the tcgen05 counterpart of causal_attention_kernel
// (cutile_gpt/kernels/attention.py:24-116).
//
// Persistent: one CTA per SM walks 128-row query tiles (heaviest causal
// spans first). Warp 9 lane 0 streams Q / K / V by TMA (3-stage K/V ring,
// double-buffered Q: the next tile's Q is loaded while the current tile
// runs); warp 8 lane 0 issues the MMAs into double-buffered S / P / O; warps
// 0-7 do the softmax, query row r owned by threads r and r + 128 (TMEM lane
// r, one half of the columns each; GPT_ATTN_SOFTMAX_WARPS=16 splits a row
// over four threads, measured slower on B200). Per key block of 128:
//   S = Q Kᵀ        tcgen05.mma M=128 N=128 K=64 into one of two TMEM S
//                   buffers; S_{j+1} is issued before the softmax of S_j
//   softmax         one tcgen05.ld pass per thread (64 scores), causal /
//                   length mask, row max shared through shared memory,
//                   P = 2^(S - m) (ex2.approx) packed bf16 into shared
//                   memory in the 128B-swizzled K-major A-operand layout
//   O_blk = P V     tcgen05.mma M=128 N=64 K=128, V read MN-major straight
//                   from its TMA tile -> TMEM columns [256,320)
//   O = O·α + O_blk in registers (α = 2^(m_old - m_new)).
// Q, K, V arrive by TMA through 4-D tensor maps {D, H, T, B} built from the
// caller's strides, so both the fused [B, T, 3C] QKV buffer and the
// [B, H, T, D] layout are read in place; rows past T are zero-filled by TMA
// and masked. K/V blocks are double-buffered by TMA.
#include "common.cuh"

namespace gpt {
namespace attn_tc {

using tc::desc_sw128;
using tc::mbar_expect_tx;
using tc::mbar_init;
using tc::mbar_wait;
using tc::smem_addr;
using tc::tc_commit;
using tc::tc_fence_after;
using tc::tc_fence_before;
using tc::tc_mma;
using tc::tmem_ld32;

constexpr int kRows = 128;   // query rows per CTA
constexpr int kKeys = 128;   // keys per block
constexpr int kD = 64;
#ifndef GPT_ATTN_SOFTMAX_WARPS
#define GPT_ATTN_SOFTMAX_WARPS 8
#endif
constexpr int kSoftmaxWarps = GPT_ATTN_SOFTMAX_WARPS;
constexpr int kThreads = (kSoftmaxWarps + 2) * 32;  // softmax warps + MMA warp + TMA warp
constexpr int kSplit = kSoftmaxWarps / 4;           // threads per query row (TMEM lane)
constexpr int kSC = 128 / kSplit;                   // score columns per thread
constexpr int kOC = 64 / kSplit;                    // output columns per thread
constexpr int kTileBytes = kRows * kD * 2;   // 16 KB (Q, K or V tile)
constexpr int kPBytes = kRows * kKeys * 2;   // 32 KB (two 64-key swizzled sub-tiles)
constexpr int kKvStages = 3;
constexpr int kQStages = 2;
constexpr int kSmem = 1024 + kQStages * kTileBytes + kKvStages * 2 * kTileBytes + 2 * kPBytes + kTileBytes + 256;

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Output tile (staged in shared memory, 128B-swizzled) -> global by TMA.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

struct Params {
  int H, T;
  int n_qblk;          // ceil(T / 128)
  int BH, n_tiles;     // B*H, B*H*n_qblk
  float scale_log2;
  __nv_bfloat16* out;
  int64_t osb, osh, ost;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void softmax_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxWarps * 32) : "memory");
}

// 32 lanes x 16 consecutive fp32 TMEM columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Walks one CTA's work: tiles t = blockIdx.x, +gridDim.x, ... (tile t = query
// block n_qblk-1 - t/(B*H) of head t%(B*H), heaviest first), and within a
// tile the causal key blocks 0..qb.
struct Cursor {
  int tile, j, nblk, qb, b, h;
  bool valid;
  __device__ void set(int t, const Params& p) {
    tile = t;
    j = 0;
    valid = t < p.n_tiles;
    if (valid) {
      qb = p.n_qblk - 1 - t / p.BH;
      const int bh = t % p.BH;
      b = bh / p.H;
      h = bh % p.H;
      nblk = qb + 1;
    }
  }
  __device__ bool last_in_tile() const { return j == nblk - 1; }
  __device__ void next(const Params& p) {
    if (++j == nblk) set(tile + (int)gridDim.x, p);
  }
};

__global__ void __launch_bounds__(kThreads, 1) attn_tc_kernel(const __grid_constant__ CUtensorMap tq,
                                                              const __grid_constant__ CUtensorMap tk,
                                                              const __grid_constant__ CUtensorMap tv,
                                                              const __grid_constant__ CUtensorMap to,
                                                              const Params p) {
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smem_dyn + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = base;                            // [2][16 KB]: Q of this tile and the next
  uint8_t* sK = sQ + kQStages * kTileBytes;      // [kKvStages][16 KB]
  uint8_t* sV = sK + kKvStages * kTileBytes;     // [kKvStages][16 KB]
  uint8_t* sP = sV + kKvStages * kTileBytes;     // [2][32 KB]: keys 0-63 | keys 64-127
  uint8_t* sO = sP + 2 * kPBytes;                // [16 KB]: output tile staged for the TMA store
  uint64_t* bars = (uint64_t*)(sO + kTileBytes);
  uint64_t* q_full = bars;                       // 2 (TMA tx)
  uint64_t* q_empty = bars + 2;                  // 2 (commit after a tile's last S)
  uint64_t* kv_full = bars + 4;                  // kKvStages (TMA tx)
  uint64_t* kv_empty = kv_full + kKvStages;      // kKvStages (commit after PV)
  uint64_t* s_full = kv_empty + kKvStages;       // 2 (commit after S)
  uint64_t* s_free = s_full + 2;                 // 2 (softmax warps)
  uint64_t* p_full = s_free + 2;                 // 2 (softmax warps)
  uint64_t* o_full = p_full + 2;                 // 2 (commit after PV)
  uint64_t* o_free = o_full + 2;                 // 2 (softmax warps)
  uint32_t* tmem_slot = (uint32_t*)(o_free + 2);
  __shared__ float sm_red[2][kSplit][kRows];   // row-max exchange, by block parity
  __shared__ float sm_l[kSplit][kRows];        // row-sum exchange at the end of a tile

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kQStages; ++i) {
      mbar_init(smem_addr(&q_full[i]), 1);
      mbar_init(smem_addr(&q_empty[i]), 1);
    }
    for (int i = 0; i < kKvStages; ++i) {
      mbar_init(smem_addr(&kv_full[i]), 1);
      mbar_init(smem_addr(&kv_empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&s_full[i]), 1);
      mbar_init(smem_addr(&o_full[i]), 1);
      mbar_init(smem_addr(&s_free[i]), kSoftmaxWarps);
      mbar_init(smem_addr(&p_full[i]), kSoftmaxWarps);
      mbar_init(smem_addr(&o_free[i]), kSoftmaxWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(512u));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;              // S buffers at columns 0 / 128, O buffers at 256 / 320
  pdl_wait();
  pdl_trigger();
  bool ok = true;

  if (warp == kSoftmaxWarps + 1) {
    // ------------------------------------------------ TMA producer (one lane)
    // Q of a tile (two slots: the next tile's Q arrives while the current tile
    // runs) and the K/V blocks (kKvStages-deep ring), in the MMA order.
    if (lane == 0) {
      Cursor lc;
      lc.set(blockIdx.x, p);
      int lg = 0, ql = 0;
      while (lc.valid && ok) {
        if (lc.j == 0) {
          const int slot = ql & 1;
          if (ql >= kQStages && !mbar_wait(smem_addr(&q_empty[slot]), (uint32_t)(((ql / kQStages) - 1) & 1))) {
            ok = false;
            break;
          }
          mbar_expect_tx(smem_addr(&q_full[slot]), kTileBytes);
          tma_load_4d(smem_addr(sQ + slot * kTileBytes), &tq, smem_addr(&q_full[slot]), 0, lc.h, lc.qb * kRows,
                      lc.b);
          ++ql;
        }
        const int st = lg % kKvStages;
        if (lg >= kKvStages && !mbar_wait(smem_addr(&kv_empty[st]), (uint32_t)(((lg / kKvStages) - 1) & 1))) {
          ok = false;
          break;
        }
        const uint32_t fb = smem_addr(&kv_full[st]);
        mbar_expect_tx(fb, 2 * kTileBytes);
        tma_load_4d(smem_addr(sK + st * kTileBytes), &tk, fb, 0, lc.h, lc.j * kKeys, lc.b);
        tma_load_4d(smem_addr(sV + st * kTileBytes), &tv, fb, 0, lc.h, lc.j * kKeys, lc.b);
        lc.next(p);
        ++lg;
      }
    }
  } else if (warp == kSoftmaxWarps) {
    // ------------------------------------------------ MMA issuer (one lane)
    if (lane == 0) {
      // kind::f16, D fp32, A/B bf16; S: both K-major, N=128; PV: B MN-major (bit 16), N=64.
      constexpr uint32_t idS = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kKeys >> 3) << 17) |
                               ((uint32_t)(kRows >> 4) << 24);
      constexpr uint32_t idO = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(kD >> 3) << 17) |
                               ((uint32_t)(kRows >> 4) << 24);
      Cursor sc, pc;                     // S-issue and PV-issue cursors
      sc.set(blockIdx.x, p);
      pc.set(blockIdx.x, p);
      int sg = 0, pg = 0, qs = 0;        // S blocks, PV blocks, tiles whose S started
      auto issue_s = [&]() {
        const int st = sg % kKvStages;
        if (sc.j == 0) {
          if (ok && !mbar_wait(smem_addr(&q_full[qs & 1]), (uint32_t)((qs / kQStages) & 1))) ok = false;
          ++qs;
        }
        const int qslot = (qs - 1) & 1;  // this tile's Q slot
        if (ok && !mbar_wait(smem_addr(&kv_full[st]), (uint32_t)((sg / kKvStages) & 1))) ok = false;
        if (ok && !mbar_wait(smem_addr(&s_free[sg & 1]), (uint32_t)(((sg >> 1) & 1) ^ 1))) ok = false;
        if (ok) {
          tc_fence_after();
          const uint64_t qd = desc_sw128(smem_addr(sQ + qslot * kTileBytes));
          const uint64_t kd = desc_sw128(smem_addr(sK + st * kTileBytes));
#pragma unroll
          for (int k = 0; k < kD / 16; ++k)
            tc_mma(tmem + (uint32_t)((sg & 1) * 128), qd + (uint64_t)(2 * k), kd + (uint64_t)(2 * k), idS, k > 0);
        }
        tc_commit(smem_addr(&s_full[sg & 1]));
        if (sc.last_in_tile()) tc_commit(smem_addr(&q_empty[qslot]));   // Q slot free once these MMAs retire
        sc.next(p);
        ++sg;
      };
      if (sc.valid) issue_s();
      while (pc.valid) {
        if (sc.valid) issue_s();         // the next S overlaps the softmax of block pg
        if (ok && !mbar_wait(smem_addr(&p_full[pg & 1]), (uint32_t)((pg >> 1) & 1))) ok = false;
        if (ok && !mbar_wait(smem_addr(&o_free[pg & 1]), (uint32_t)(((pg >> 1) & 1) ^ 1))) ok = false;
        const int st = pg % kKvStages;
        if (ok) {
          tc_fence_after();
          const uint64_t vd = desc_sw128(smem_addr(sV + st * kTileBytes));
          const uint32_t pbase = smem_addr(sP + (pg & 1) * kPBytes);
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk) {
            const uint64_t pd = desc_sw128(pbase + (uint32_t)((kk >> 2) * (kRows * 128))) + (uint64_t)(2 * (kk & 3));
            tc_mma(tmem + 256 + (uint32_t)((pg & 1) * 64), pd, vd + (uint64_t)(kk * 128), idO, kk > 0);  // +16 keys
          }
        }
        tc_commit(smem_addr(&o_full[pg & 1]));
        tc_commit(smem_addr(&kv_empty[st]));
        pc.next(p);
        ++pg;
      }
    }
  } else {
    // ------------------------------------------------ softmax: threads r, r+128, ... share query row r
    static_assert((kSC == 32 && kOC == 16) || (kSC == 64 && kOC == 32), "2 or 4 threads per query row");
    const int rl = tid & (kRows - 1);
    const int part = tid >> 7;                       // this thread's quarter of the keys / O columns
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    int g = 0;   // global block counter (same order as the producer)
    for (int t = blockIdx.x; t < p.n_tiles; t += gridDim.x) {
      Cursor c;
      c.set(t, p);
      const int row = c.qb * kRows + rl;
      float o[kOC];
#pragma unroll
      for (int d = 0; d < kOC; ++d) o[d] = 0.f;
      float m_run = -INFINITY, l_part = 0.f, alpha_prev = 1.f;
      // O_i (relative to m_i) folded into o (relative to m_{i-1}) with alpha_i.
      auto fold_o = [&](int gi, float alpha_i) {
        if (!mbar_wait(smem_addr(&o_full[gi & 1]), (uint32_t)((gi >> 1) & 1))) ok = false;
        tc_fence_after();
        uint32_t r[kOC];
        if constexpr (kOC == 16)
          tmem_ld16(tmem + 256 + (uint32_t)((gi & 1) * 64 + part * kOC) + lane_off, r);
        else
          tmem_ld32(tmem + 256 + (uint32_t)((gi & 1) * 64 + part * kOC) + lane_off, r);
#pragma unroll
        for (int d = 0; d < kOC; ++d) o[d] = o[d] * alpha_i + __uint_as_float(r[d]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(smem_addr(&o_free[gi & 1]));
      };
      for (int j = 0; j < c.nblk; ++j, ++g) {
        if (!mbar_wait(smem_addr(&s_full[g & 1]), (uint32_t)((g >> 1) & 1))) ok = false;
        tc_fence_after();
        const int kbase = j * kKeys + part * kSC;
        const bool diag = (j == c.nblk - 1);
        float sv[kSC];
#pragma unroll
        for (int c2 = 0; c2 < kSC; c2 += 32) {
          uint32_t r[32];
          tmem_ld32(tmem + (uint32_t)((g & 1) * 128 + part * kSC + c2) + lane_off, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[c2 + i] = __uint_as_float(r[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(smem_addr(&s_free[g & 1]));   // S buffer may be overwritten
        // mask only where needed: the diagonal block and a block past T
        float mx = -INFINITY;
        if (diag || kbase + kSC > p.T) {
          // keys kbase .. kbase + nvalid - 1 are inside T and not after this row
          const int nvalid = min(p.T, diag ? row + 1 : p.T) - kbase;
#pragma unroll
          for (int i = 0; i < kSC; ++i) {
            if (i >= nvalid) sv[i] = -INFINITY;
            mx = fmaxf(mx, sv[i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < kSC; ++i) mx = fmaxf(mx, sv[i]);
        }
        sm_red[g & 1][part][rl] = mx * p.scale_log2;   // scale > 0 commutes with max
        softmax_bar();
        mx = m_run;
#pragma unroll
        for (int s2 = 0; s2 < kSplit; ++s2) mx = fmaxf(mx, sm_red[g & 1][s2][rl]);
        const float mref = mx == -INFINITY ? 0.f : mx;
        const float alpha = ex2(m_run - mref);
        float rs = 0.f;
        // keys [part*kSC, +kSC): sub-tile (part*kSC)/64 (64 keys, 128B-swizzled
        // K-major rows), 16-byte chunks from ((part*kSC) % 64) / 8 of row rl
        uint8_t* prow = sP + (g & 1) * kPBytes + ((part * kSC) >> 6) * (kRows * 128) + rl * 128;
#pragma unroll
        for (int q = 0; q < kSC / 8; ++q) {
          uint32_t w[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float p0 = ex2(fmaf(sv[8 * q + 2 * u], p.scale_log2, -mref));
            const float p1 = ex2(fmaf(sv[8 * q + 2 * u + 1], p.scale_log2, -mref));
            rs += p0 + p1;
            __nv_bfloat162 bp = __floats2bfloat162_rn(p0, p1);
            w[u] = *reinterpret_cast<uint32_t*>(&bp);
          }
          const int chunk = ((part * kSC) & 63) / 8 + q;
          *reinterpret_cast<uint4*>(prow + ((chunk ^ (rl & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        l_part = l_part * alpha + rs;
        m_run = mx;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P visible to the MMA
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(smem_addr(&p_full[g & 1]));
        if (j > 0) fold_o(g - 1, alpha_prev);
        alpha_prev = alpha;
      }
      fold_o(g - 1, alpha_prev);
      // row sum across the parts (sm_l is written again only after the next
      // tile's block barriers, which every reader passes first)
      sm_l[part][rl] = l_part;
      // the previous tile's TMA store has finished reading sO before it is rewritten
      if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      softmax_bar();
      float lsum = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < kSplit; ++s2) lsum += sm_l[s2][rl];
      {
        // row rl, columns [part*kOC, +kOC) -> 16-byte chunks of the 128-byte
        // row, XOR-swizzled by (row & 7) as the tensor map expects
        const float inv = __fdividef(1.f, lsum);
        uint8_t* srow = sO + rl * 128;
#pragma unroll
        for (int v = 0; v < kOC / 8; ++v) {
          uint32_t w[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            __nv_bfloat162 tt = __floats2bfloat162_rn(o[8 * v + 2 * u] * inv, o[8 * v + 2 * u + 1] * inv);
            w[u] = *reinterpret_cast<uint32_t*>(&tt);
          }
          const int chunk = (part * kOC) / 8 + v;
          *reinterpret_cast<uint4*>(srow + ((chunk ^ (rl & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        softmax_bar();
        if (tid == 0 && ok) {  // rows past T are clipped by the tensor map
          tma_store_4d(&to, smem_addr(sO), 0, c.h, c.qb * kRows, c.b);
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        (void)row;
      }
    }
  }
  if (tid == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // output tiles written
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u));
  }
}

// 4-D map {D, H, T, B} over a bf16 tensor with element strides (sb, sh, st),
// box {64, 1, 128, 1}, 128-byte swizzle, rows past T zero-filled.
static int make_map4(CUtensorMap* map, const void* ptr, int64_t B, int64_t H, int64_t T, int64_t sb, int64_t sh,
                     int64_t st) {
  auto enc = tc::get_encode();
  if (!enc) return fail(GPT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(sh * 2), (cuuint64_t)(st * 2), (cuuint64_t)(sb * 2)};
  cuuint32_t box[4] = {(cuuint32_t)kD, 1, (cuuint32_t)kRows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GPT_ERR_CUDA, "cuTensorMapEncodeTiled (attention) failed (%d)", (int)r);
  return GPT_OK;
}

// Whether the tcgen05 kernel serves these strides (D = 64, 16-byte strides, T < 2^31).
inline bool eligible(int64_t D, const void* q, const void* k, const void* v, const void* o, const int64_t* qs,
                     const int64_t* ks, const int64_t* vs, const int64_t* os) {
  if (D != kD) return false;
  for (const void* ptr : {q, k, v, o})
    if (!aligned(ptr, 16)) return false;
  for (const int64_t* s : {qs, ks, vs, os})
    for (int i = 0; i < 3; ++i)
      if (s[i] % 8 != 0 || s[i] <= 0) return false;
  return true;
}

int launch(const void* q, const void* k, const void* v, void* out, int64_t B, int64_t H, int64_t T,
           const int64_t* qs, const int64_t* ks, const int64_t* vs, const int64_t* os, float scale_log2,
           cudaStream_t st) {
  CUtensorMap mq, mk, mv, mo;
  int s = make_map4(&mq, q, B, H, T, qs[0], qs[1], qs[2]);
  if (!s) s = make_map4(&mk, k, B, H, T, ks[0], ks[1], ks[2]);
  if (!s) s = make_map4(&mv, v, B, H, T, vs[0], vs[1], vs[2]);
  if (!s) s = make_map4(&mo, out, B, H, T, os[0], os[1], os[2]);
  if (s) return s;
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> g(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
      if (e != cudaSuccess) return fail(GPT_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      done[dev] = true;
    }
  }
  Params p;
  p.H = (int)H;
  p.T = (int)T;
  p.n_qblk = (int)((T + kRows - 1) / kRows);
  p.scale_log2 = scale_log2;
  p.out = (__nv_bfloat16*)out;
  p.osb = os[0];
  p.osh = os[1];
  p.ost = os[2];
  const int64_t tiles = B * H * p.n_qblk;
  if (tiles > 0x7fffffff) return fail(GPT_ERR_UNSUPPORTED, "attention work too large");
  p.BH = (int)(B * H);
  p.n_tiles = (int)tiles;
  int sms = device_sm_count();
  if (sms <= 0) sms = 148;
  const int grid = (int)(tiles < sms ? tiles : sms);   // persistent: one CTA per SM
  launch_pdl(attn_tc_kernel, dim3((unsigned)grid), dim3(kThreads), kSmem, st, mq, mk, mv, mo, p);
  return launch_status("attention_tc");
}

}  // namespace attn_tc
}  // namespace gpt
