// Causal prefill attention on the 5th-generation tensor cores (bf16,
// head_dim 64), the tcgen05 counterpart of causal_attention_kernel
// (cutile_gpt/kernels/attention.py:24-116).
//
// Persistent: one CTA per SM walks 128-row query tiles (heaviest causal
// spans first). Warp 8 lane 0 is the TMA producer and MMA issuer, running
// ahead through a 3-stage K/V ring and double-buffered S / P / O; warps 0-7
// do the softmax, query row r owned by threads r and r + 128 (TMEM lane r,
// one half of the columns each). Per key block of 128:
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
constexpr int kSoftmaxWarps = 8;
constexpr int kThreads = (kSoftmaxWarps + 1) * 32;  // 8 softmax warps + producer/MMA warp
constexpr int kTileBytes = kRows * kD * 2;   // 16 KB (Q, K or V tile)
constexpr int kPBytes = kRows * kKeys * 2;   // 32 KB (two 64-key swizzled sub-tiles)
constexpr int kKvStages = 3;
constexpr int kSmem = 1024 + kTileBytes + kKvStages * 2 * kTileBytes + 2 * kPBytes + 256;

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
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

__device__ __forceinline__ void softmax_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

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
                                                              const Params p) {
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smem_dyn + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = base;
  uint8_t* sK = sQ + kTileBytes;                 // [3][16 KB]
  uint8_t* sV = sK + kKvStages * kTileBytes;     // [3][16 KB]
  uint8_t* sP = sV + kKvStages * kTileBytes;     // [2][32 KB]: keys 0-63 | keys 64-127
  uint64_t* bars = (uint64_t*)(sP + 2 * kPBytes);
  uint64_t* q_full = bars;                       // 1 (TMA tx)
  uint64_t* q_empty = bars + 1;                  // 1 (commit after a tile's last S)
  uint64_t* kv_full = bars + 2;                  // 3 (TMA tx)
  uint64_t* kv_empty = bars + 5;                 // 3 (commit after PV)
  uint64_t* s_full = bars + 8;                   // 2 (commit after S)
  uint64_t* s_free = bars + 10;                  // 2 (8 softmax warps)
  uint64_t* p_full = bars + 12;                  // 2 (8 softmax warps)
  uint64_t* o_full = bars + 14;                  // 2 (commit after PV)
  uint64_t* o_free = bars + 16;                  // 2 (8 softmax warps)
  uint32_t* tmem_slot = (uint32_t*)(bars + 18);
  __shared__ float sm_red[2][2][kRows];   // row-max exchange, by block parity
  __shared__ float sm_l[2][kRows];        // row-sum exchange at the end of a tile

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    mbar_init(smem_addr(q_full), 1);
    mbar_init(smem_addr(q_empty), 1);
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

  if (warp == kSoftmaxWarps) {
    // ------------------------------------------------ TMA producer + MMA issuer (one lane)
    if (lane == 0) {
      // kind::f16, D fp32, A/B bf16; S: both K-major, N=128; PV: B MN-major (bit 16), N=64.
      constexpr uint32_t idS = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kKeys >> 3) << 17) |
                               ((uint32_t)(kRows >> 4) << 24);
      constexpr uint32_t idO = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(kD >> 3) << 17) |
                               ((uint32_t)(kRows >> 4) << 24);
      Cursor lc, sc, pc;                 // load, S-issue and PV-issue cursors
      lc.set(blockIdx.x, p);
      sc.set(blockIdx.x, p);
      pc.set(blockIdx.x, p);
      int lg = 0, sg = 0, pg = 0;        // global block counters of the three cursors
      int qtiles = 0;                    // Q tiles loaded so far
      auto load_kv = [&]() {             // next K/V block into its ring stage
        const int st = lg % kKvStages;
        if (lg >= kKvStages && ok && !mbar_wait(smem_addr(&kv_empty[st]), (uint32_t)(((lg / kKvStages) - 1) & 1)))
          ok = false;
        const uint32_t fb = smem_addr(&kv_full[st]);
        mbar_expect_tx(fb, 2 * kTileBytes);
        tma_load_4d(smem_addr(sK + st * kTileBytes), &tk, fb, 0, lc.h, lc.j * kKeys, lc.b);
        tma_load_4d(smem_addr(sV + st * kTileBytes), &tv, fb, 0, lc.h, lc.j * kKeys, lc.b);
        lc.next(p);
        ++lg;
      };
      auto load_q = [&](const Cursor& c) {
        if (qtiles > 0 && ok && !mbar_wait(smem_addr(q_empty), (uint32_t)((qtiles - 1) & 1))) ok = false;
        mbar_expect_tx(smem_addr(q_full), kTileBytes);
        tma_load_4d(smem_addr(sQ), &tq, smem_addr(q_full), 0, c.h, c.qb * kRows, c.b);
        ++qtiles;
      };
      auto issue_s = [&]() {
        const int st = sg % kKvStages;
        if (sc.j == 0) {
          load_q(sc);
          if (ok && !mbar_wait(smem_addr(q_full), (uint32_t)((qtiles - 1) & 1))) ok = false;
        }
        if (ok && !mbar_wait(smem_addr(&kv_full[st]), (uint32_t)((sg / kKvStages) & 1))) ok = false;
        if (ok && !mbar_wait(smem_addr(&s_free[sg & 1]), (uint32_t)(((sg >> 1) & 1) ^ 1))) ok = false;
        if (ok) {
          tc_fence_after();
          const uint64_t qd = desc_sw128(smem_addr(sQ));
          const uint64_t kd = desc_sw128(smem_addr(sK + st * kTileBytes));
#pragma unroll
          for (int k = 0; k < kD / 16; ++k)
            tc_mma(tmem + (uint32_t)((sg & 1) * 128), qd + (uint64_t)(2 * k), kd + (uint64_t)(2 * k), idS, k > 0);
        }
        tc_commit(smem_addr(&s_full[sg & 1]));
        if (sc.last_in_tile()) tc_commit(smem_addr(q_empty));   // Q may be replaced once these MMAs retire
        sc.next(p);
        ++sg;
      };
      for (int i = 0; i < kKvStages && lc.valid; ++i) load_kv();
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
        if (lc.valid) load_kv();         // waits for this stage's PV, then refills it
      }
    }
  } else {
    // ------------------------------------------------ softmax: threads r and r+128 share query row r
    const int rl = tid & (kRows - 1);
    const int half = tid >> 7;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    int g = 0;   // global block counter (same order as the producer)
    for (int t = blockIdx.x; t < p.n_tiles; t += gridDim.x) {
      Cursor c;
      c.set(t, p);
      const int row = c.qb * kRows + rl;
      float o[32];
#pragma unroll
      for (int d = 0; d < 32; ++d) o[d] = 0.f;
      float m_run = -INFINITY, l_part = 0.f, alpha_prev = 1.f;
      // O_i (relative to m_i) folded into o (relative to m_{i-1}) with alpha_i.
      auto fold_o = [&](int gi, float alpha_i) {
        if (!mbar_wait(smem_addr(&o_full[gi & 1]), (uint32_t)((gi >> 1) & 1))) ok = false;
        tc_fence_after();
        uint32_t r[32];
        tmem_ld32(tmem + 256 + (uint32_t)((gi & 1) * 64 + half * 32) + lane_off, r);
#pragma unroll
        for (int d = 0; d < 32; ++d) o[d] = o[d] * alpha_i + __uint_as_float(r[d]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(smem_addr(&o_free[gi & 1]));
      };
      for (int j = 0; j < c.nblk; ++j, ++g) {
        if (!mbar_wait(smem_addr(&s_full[g & 1]), (uint32_t)((g >> 1) & 1))) ok = false;
        tc_fence_after();
        const int kbase = j * kKeys + half * 64;
        const bool diag = (j == c.nblk - 1);
        float sv[64];
        {
          uint32_t r[32];
          tmem_ld32(tmem + (uint32_t)((g & 1) * 128 + half * 64) + lane_off, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[i] = __uint_as_float(r[i]);
          tmem_ld32(tmem + (uint32_t)((g & 1) * 128 + half * 64 + 32) + lane_off, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[32 + i] = __uint_as_float(r[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(smem_addr(&s_free[g & 1]));   // S buffer may be overwritten
        // mask only where needed: the diagonal block and a block past T
        float mx = -INFINITY;
        if (diag || kbase + 64 > p.T) {
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const int key = kbase + i;
            if (!(key < p.T && (!diag || key <= row))) sv[i] = -INFINITY;
            mx = fmaxf(mx, sv[i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) mx = fmaxf(mx, sv[i]);
        }
        sm_red[g & 1][half][rl] = mx * p.scale_log2;   // scale > 0 commutes with max
        softmax_bar();
        mx = fmaxf(m_run, fmaxf(sm_red[g & 1][0][rl], sm_red[g & 1][1][rl]));
        const float mref = mx == -INFINITY ? 0.f : mx;
        const float alpha = ex2(m_run - mref);
        float rs = 0.f;
        uint8_t* prow = sP + (g & 1) * kPBytes + half * (kRows * 128) + rl * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {   // 8 chunks of 8 keys, 128B-swizzled K-major rows
          uint32_t w[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float p0 = ex2(fmaf(sv[8 * q + 2 * u], p.scale_log2, -mref));
            const float p1 = ex2(fmaf(sv[8 * q + 2 * u + 1], p.scale_log2, -mref));
            rs += p0 + p1;
            __nv_bfloat162 bp = __floats2bfloat162_rn(p0, p1);
            w[u] = *reinterpret_cast<uint32_t*>(&bp);
          }
          *reinterpret_cast<uint4*>(prow + ((q ^ (rl & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
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
      // row sum across the two halves (sm_l is written again only after the
      // next tile's block barriers, which every reader passes first)
      sm_l[half][rl] = l_part;
      softmax_bar();
      const float lsum = sm_l[0][rl] + sm_l[1][rl];
      if (ok && row < p.T) {
        const float inv = 1.f / lsum;
        __nv_bfloat16* dst =
            p.out + (int64_t)c.b * p.osb + (int64_t)c.h * p.osh + (int64_t)row * p.ost + half * 32;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t w[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            __nv_bfloat162 tt = __floats2bfloat162_rn(o[8 * v + 2 * u] * inv, o[8 * v + 2 * u + 1] * inv);
            w[u] = *reinterpret_cast<uint32_t*>(&tt);
          }
          *reinterpret_cast<uint4*>(dst + 8 * v) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  }
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
  CUtensorMap mq, mk, mv;
  int s = make_map4(&mq, q, B, H, T, qs[0], qs[1], qs[2]);
  if (!s) s = make_map4(&mk, k, B, H, T, ks[0], ks[1], ks[2]);
  if (!s) s = make_map4(&mv, v, B, H, T, vs[0], vs[1], vs[2]);
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
  launch_pdl(attn_tc_kernel, dim3((unsigned)grid), dim3(kThreads), kSmem, st, mq, mk, mv, p);
  return launch_status("attention_tc");
}

}  // namespace attn_tc
}  // namespace gpt
