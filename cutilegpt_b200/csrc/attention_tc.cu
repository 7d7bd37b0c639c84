// Causal prefill attention on the 5th-generation tensor cores (bf16,
// head_dim 64), the tcgen05 counterpart of causal_attention_kernel
// (cutile_gpt/kernels/attention.py:24-116).
//
// Persistent, one CTA per SM, two independent pipelines per CTA: pipeline s
// (s = 0, 1) walks its own 128-row query tiles (heaviest causal spans
// first), with its own TMA producer lane (warp 10 + s), MMA issuer lane
// (warp 8 + s) and softmax warpgroup (warps 4s .. 4s+3, one thread per query
// row = TMEM lane). The two pipelines share the tensor core, so one tile's
// MMAs run while the other tile's softmax does its exponentials. Per key
// block of 128:
//   S = Q Kᵀ      tcgen05.mma M=128 N=128 K=64 -> TMEM (this pipeline's S)
//   softmax       the thread's whole S row (128 columns) is read into
//                 registers once, which frees S for the next block's QKᵀ at
//                 once; row max, P = 2^(S·scale - m) (ex2.approx), row sum,
//                 P packed bf16 into TMEM (tcgen05.st), masked keys -> 0
//   O += P V      tcgen05.mma with A = P from TMEM, B = V MN-major from its
//                 TMA tile, accumulating in TMEM across the tile's blocks
// The running max m only moves when a block's max exceeds it by more than
// 2^8 (log2 domain): then O in TMEM and the row sum are rescaled once;
// otherwise P uses the stale m (values stay below 2^8), and the final O / l
// is the same softmax. K and V blocks have separate two-slot rings (a K slot
// is released by the QKᵀ that read it, a V slot by the PV). TMEM per pipeline: S 128 columns, P 64, O 64 (512 in
// all). Q, K, V arrive by TMA through 4-D tensor maps {D, H, T, B} built
// from the caller's strides, so both the fused [B, T, 3C] QKV buffer and the
// [B, H, T, D] layout are read in place; rows past T are zero-filled by TMA
// and masked; the output tile leaves through a TMA store (rows past T
// clipped). Every wait is bounded.
#include <map>
#include <memory>
#include <queue>
#include <tuple>
#include <vector>

#include "common.cuh"

namespace gpt {
namespace attn_tc {

using tc::desc_sw128;
using tc::mbar_arrive;
using tc::mbar_expect_tx;
using tc::mbar_init;
using tc::mbar_wait;
using tc::smem_addr;
using tc::tc_commit;
using tc::tc_fence_after;
using tc::tc_fence_before;
using tc::tc_mma;
using tc::tmem_ld32;

constexpr int kRows = 128;   // query rows per tile
constexpr int kKeys = 128;   // keys per block
constexpr int kD = 64;
constexpr int kPipes = 2;
constexpr int kThreads = (4 * kPipes + 2 * kPipes) * 32;   // softmax warpgroups + MMA + TMA warps
constexpr int kTileBytes = kRows * kD * 2;   // 16 KB (Q, K, V or output tile)
constexpr int kKvStages = 2;
constexpr int kQStages = 2;
constexpr int kPipeBytes = kQStages * kTileBytes + kKvStages * 2 * kTileBytes + kTileBytes;   // 112 KB
constexpr int kSmem = 1024 + kPipes * kPipeBytes + 512;
constexpr float kRescale = 8.f;   // log2 of the largest P value allowed before O is rescaled

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
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed f32x2 arithmetic (sm_100): two lanes per instruction.
__device__ __forceinline__ uint64_t pack_f2(float a, float b) {
  uint64_t v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(a), "f"(b));
  return v;
}
__device__ __forceinline__ uint64_t pack_u2(uint32_t a, uint32_t b) {
  uint64_t v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "r"(a), "r"(b));
  return v;
}
__device__ __forceinline__ void unpack_f2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// O += P V with P (bf16, M = 128 x K = 16 slice) read from TMEM.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accum));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  tmem_st16(taddr, r);
  tmem_st16(taddr + 16, r + 16);
}
__device__ __forceinline__ void tmem_ld32_nw(uint32_t taddr, uint32_t* r) {   // no wait::ld
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Bounded wait for the phase of the turn barrier, or until the other
// pipeline has finished all its work (it then arrives no more).
__device__ __noinline__ bool turn_wait(uint32_t bar, uint32_t parity, const volatile uint32_t* other_done) {
  uint64_t t0 = 0;
  for (int it = 0;; ++it) {
    if (tc::mbar_try(bar, parity)) return true;
    if (*other_done) return true;
    if ((it & 31) == 31) {
      const uint64_t t = global_timer_ns();
      if (t0 == 0) {
        t0 = t;
      } else if (t - t0 > g_wait_limit_ns) {
        record_device_error(GPT_DEVERR_TIMEOUT);
        return false;
      }
    }
  }
}
// Named barrier of one softmax warpgroup (ids 1, 2).
__device__ __forceinline__ void wg_bar(int pipe) {
  asm volatile("bar.sync %0, 128;" ::"r"(1 + pipe) : "memory");
}

// Tile schedule: tile t is query block n_qblk-1 - t/(B*H) of head t%(B*H), so
// tiles are numbered heaviest first (a tile costs its number of causal key
// blocks). When the problem is small enough the host assigns the tiles to the
// pipelines by longest-processing-time-first (each tile, heaviest first, to
// the pipeline with the least work so far) and passes the lists here:
// v[q] .. v[q+1]-1 index the tile ids of pipeline q in v[n_pipes + 1 + ...].
// Otherwise (n == 0) pipeline q takes tiles q, q + n_pipes, q + 2 n_pipes, ...
constexpr int kSchedMax = 4096;
struct Sched {
  int n;   // entries used in v (0: strided assignment)
  uint16_t v[kSchedMax];
};

// Walks one pipeline's work, and within a tile the causal key blocks 0..qb.
struct Cursor {
  int tile, j, nblk, qb, b, h;
  int k, kend, q, n_pipes;
  const uint16_t* list;
  bool valid;
  __device__ void start(int pipe_id, int pipes, const Params& p, const Sched& s) {
    q = pipe_id;
    n_pipes = pipes;
    if (s.n > 0) {
      list = s.v + pipes + 1;
      k = s.v[pipe_id];
      kend = s.v[pipe_id + 1];
    } else {
      list = nullptr;
      k = 0;
      kend = 0x7fffffff;
    }
    load(p);
  }
  __device__ void load(const Params& p) {
    j = 0;
    tile = list ? (k < kend ? (int)list[k] : p.n_tiles) : q + k * n_pipes;
    valid = tile < p.n_tiles;
    if (valid) {
      qb = p.n_qblk - 1 - tile / p.BH;
      const int bh = tile % p.BH;
      b = bh / p.H;
      h = bh % p.H;
      nblk = qb + 1;
    }
  }
  __device__ bool last_in_tile() const { return j == nblk - 1; }
  __device__ void next_tile(const Params& p) {
    ++k;
    load(p);
  }
  __device__ void next(const Params& p) {
    if (++j == nblk) next_tile(p);
  }
};

__global__ void __launch_bounds__(kThreads, 1) attn_tc_kernel(const __grid_constant__ CUtensorMap tq,
                                                              const __grid_constant__ CUtensorMap tk,
                                                              const __grid_constant__ CUtensorMap tv,
                                                              const __grid_constant__ CUtensorMap to,
                                                              const Params p,
                                                              const __grid_constant__ Sched sched) {
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smem_dyn + 1023) & ~(uintptr_t)1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // role and pipeline of this warp
  const int pipe = warp < 4 * kPipes ? warp / 4 : (warp - 4 * kPipes) % kPipes;
  uint8_t* pb = base + pipe * kPipeBytes;
  uint8_t* sQ = pb;                                // [2][16 KB]
  uint8_t* sK = sQ + kQStages * kTileBytes;        // [kKvStages][16 KB]
  uint8_t* sV = sK + kKvStages * kTileBytes;       // [kKvStages][16 KB]
  uint8_t* sO = sV + kKvStages * kTileBytes;       // [16 KB] output staging
  uint64_t* bars = (uint64_t*)(base + kPipes * kPipeBytes) + pipe * 24;
  uint64_t* q_full = bars;                         // 2 (TMA tx)
  uint64_t* q_empty = bars + 2;                    // 2 (commit after a tile's last S)
  uint64_t* k_full = bars + 4;                     // kKvStages (TMA tx)
  uint64_t* k_empty = bars + 4 + kKvStages;        // kKvStages (commit after S)
  uint64_t* v_full = bars + 4 + 2 * kKvStages;     // kKvStages (TMA tx)
  uint64_t* v_empty = bars + 4 + 3 * kKvStages;    // kKvStages (commit after PV)
  uint64_t* s_full = bars + 4 + 4 * kKvStages;     // commit after S
  uint64_t* s_free = s_full + 1;                   // softmax warps: S read
  uint64_t* p_full = s_full + 2;                   // softmax warps: P written (and O rescaled)
  uint64_t* o_full = s_full + 3;                   // commit after PV
  uint64_t* o_free = s_full + 4;                   // softmax warps: final O read
  uint64_t* turn_mine = s_full + 5;                // the other pipeline's exponentials are done
  uint64_t* turn_other = (uint64_t*)(base + kPipes * kPipeBytes) + (1 - pipe) * 24 + 4 + 4 * kKvStages + 5;
  uint32_t* tmem_slot = (uint32_t*)((uint64_t*)(base + kPipes * kPipeBytes) + kPipes * 24);
  volatile uint32_t* pipe_done = tmem_slot + 1;    // [kPipes]: a pipeline's softmax has finished

  if (tid == 0) {
    for (int q = 0; q < kPipes; ++q) {
      uint64_t* bq = (uint64_t*)(base + kPipes * kPipeBytes) + q * 24;
      for (int i = 0; i < 4 + 4 * kKvStages; ++i) mbar_init(smem_addr(&bq[i]), 1);
      uint64_t* sf = bq + 4 + 4 * kKvStages;
      mbar_init(smem_addr(&sf[0]), 1);   // s_full
      mbar_init(smem_addr(&sf[1]), 4);   // s_free
      mbar_init(smem_addr(&sf[2]), 4);   // p_full
      mbar_init(smem_addr(&sf[3]), 1);   // o_full
      mbar_init(smem_addr(&sf[4]), 4);   // o_free
      mbar_init(smem_addr(&sf[5]), 4);   // turn
    }
    pipe_done[0] = 0;
    pipe_done[1] = 0;
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
  // this pipeline's TMEM: S at +0 (128 columns), P at +128 (64), O at +192 (64)
  const uint32_t tm = *tmem_slot + (uint32_t)(pipe * 256);
  pdl_wait();
  pdl_trigger();
  bool ok = true;
  const int pipe_id = kPipes * (int)blockIdx.x + pipe, n_pipes = kPipes * (int)gridDim.x;

  if (warp >= 4 * kPipes + kPipes) {
    // ------------------------------------------------ TMA producer (one lane per pipeline)
    if (lane == 0) {
      Cursor lc;
      lc.start(pipe_id, n_pipes, p, sched);
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
        // K and V have separate rings: a K slot is free once its QKᵀ has run, well before the PV
        // that frees the V slot, so the next K blocks arrive a softmax step earlier
        const int st = lg % kKvStages;
        const uint32_t par = (uint32_t)(((lg / kKvStages) - 1) & 1);
        if (lg >= kKvStages && !mbar_wait(smem_addr(&k_empty[st]), par)) {
          ok = false;
          break;
        }
        mbar_expect_tx(smem_addr(&k_full[st]), kTileBytes);
        tma_load_4d(smem_addr(sK + st * kTileBytes), &tk, smem_addr(&k_full[st]), 0, lc.h, lc.j * kKeys, lc.b);
        if (lg >= kKvStages && !mbar_wait(smem_addr(&v_empty[st]), par)) {
          ok = false;
          break;
        }
        mbar_expect_tx(smem_addr(&v_full[st]), kTileBytes);
        tma_load_4d(smem_addr(sV + st * kTileBytes), &tv, smem_addr(&v_full[st]), 0, lc.h, lc.j * kKeys, lc.b);
        lc.next(p);
        ++lg;
      }
    }
  } else if (warp >= 4 * kPipes) {
    // ------------------------------------------------ MMA issuer (one lane per pipeline)
    if (lane == 0) {
      // kind::f16, D fp32, A/B bf16; S: both K-major, N=128; PV: A from TMEM, B MN-major (bit 16), N=64.
      constexpr uint32_t idS = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kKeys >> 3) << 17) |
                               ((uint32_t)(kRows >> 4) << 24);
      constexpr uint32_t idO = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(kD >> 3) << 17) |
                               ((uint32_t)(kRows >> 4) << 24);
      Cursor sc, pc;                     // S-issue and PV-issue cursors
      sc.start(pipe_id, n_pipes, p, sched);
      pc.start(pipe_id, n_pipes, p, sched);
      int sg = 0, pg = 0, qs = 0, tiles_pv = 0;
      auto issue_s = [&]() {
        const int st = sg % kKvStages;
        if (sc.j == 0) {
          if (ok && !mbar_wait(smem_addr(&q_full[qs & 1]), (uint32_t)((qs / kQStages) & 1))) ok = false;
          ++qs;
        }
        const int qslot = (qs - 1) & 1;
        if (ok && !mbar_wait(smem_addr(&k_full[st]), (uint32_t)((sg / kKvStages) & 1))) ok = false;
        if (ok && sg > 0 && !mbar_wait(smem_addr(s_free), (uint32_t)((sg - 1) & 1))) ok = false;
        if (ok) {
          tc_fence_after();
          const uint64_t qd = desc_sw128(smem_addr(sQ + qslot * kTileBytes));
          const uint64_t kd = desc_sw128(smem_addr(sK + st * kTileBytes));
#pragma unroll
          for (int k = 0; k < kD / 16; ++k)
            tc_mma(tm, qd + (uint64_t)(2 * k), kd + (uint64_t)(2 * k), idS, k > 0);
        }
        tc_commit(smem_addr(s_full));
        tc_commit(smem_addr(&k_empty[st]));
        if (sc.last_in_tile()) tc_commit(smem_addr(&q_empty[qslot]));   // Q slot free once these MMAs retire
        sc.next(p);
        ++sg;
      };
      if (sc.valid) issue_s();
      while (pc.valid) {
        if (sc.valid) issue_s();         // the next S is computed while the softmax of block pg runs
        if (ok && !mbar_wait(smem_addr(p_full), (uint32_t)(pg & 1))) ok = false;
        if (pc.j == 0) {                 // a new tile overwrites O: the previous tile's O must have been read
          if (ok && tiles_pv > 0 && !mbar_wait(smem_addr(o_free), (uint32_t)((tiles_pv - 1) & 1))) ok = false;
          ++tiles_pv;
        }
        const int st = pg % kKvStages;
        if (ok && !mbar_wait(smem_addr(&v_full[st]), (uint32_t)((pg / kKvStages) & 1))) ok = false;
        if (ok) {
          tc_fence_after();
          const uint64_t vd = desc_sw128(smem_addr(sV + st * kTileBytes));
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk)   // 16 keys: 8 packed P columns, 16 V rows (2 KB)
            tc_mma_ts(tm + 192, tm + 128 + (uint32_t)(kk * 8), vd + (uint64_t)(kk * 128), idO,
                      (pc.j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(smem_addr(o_full));
        tc_commit(smem_addr(&v_empty[st]));
        pc.next(p);
        ++pg;
      }
    }
  } else {
    // ------------------------------------------------ softmax: thread = query row = TMEM lane
    const int rl = tid & (kRows - 1);
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tm + lane_off, tP = tm + 128 + lane_off, tO = tm + 192 + lane_off;
    int g = 0;       // blocks of this pipeline so far
    int n_exp = 0;   // exponential phases of this pipeline so far
    Cursor c;
    for (c.start(pipe_id, n_pipes, p, sched); c.valid; c.next_tile(p)) {
      const int row = c.qb * kRows + rl;
      float m_use = -INFINITY, l = 0.f;
      for (int j = 0; j < c.nblk; ++j, ++g) {
        if (!mbar_wait(smem_addr(s_full), (uint32_t)(g & 1))) ok = false;
        tc_fence_after();
        // the whole S row in registers: one read of TMEM, after which the next S may overwrite it
        uint32_t r[kKeys];
#pragma unroll
        for (int c2 = 0; c2 < kKeys; c2 += 32) tmem_ld32_nw(tS + (uint32_t)c2, r + c2);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(s_free));
        const int kbase = j * kKeys;
        // keys kbase .. kbase + nvalid - 1 are inside T and not after this row
        const int nvalid = min(p.T, j == c.nblk - 1 ? row + 1 : p.T) - kbase;
        if (nvalid < kKeys) {
#pragma unroll
          for (int i = 0; i < kKeys; ++i)
            if (i >= nvalid) r[i] = 0xff800000u;   // -inf: exponential 0
        }
        // row max: 8 independent chains of 3-input maxima
        float m8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = fmaxf(__uint_as_float(r[i]), __uint_as_float(r[i + 8]));
#pragma unroll
        for (int i = 16; i < kKeys; i += 16)
#pragma unroll
          for (int k = 0; k < 8; ++k) m8[k] = fmax3(m8[k], __uint_as_float(r[i + k]), __uint_as_float(r[i + 8 + k]));
        float mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        mx *= p.scale_log2;   // scale > 0 commutes with max
        bool rescale = false;
        float alpha = 1.f;
        if (j == 0) {
          m_use = mx;
        } else if (mx > m_use + kRescale) {
          alpha = ex2(m_use - mx);
          m_use = mx;
          rescale = true;
        }
        // P and O of the previous block are free once its PV has completed
        if (g > 0 && !mbar_wait(smem_addr(o_full), (uint32_t)((g - 1) & 1))) ok = false;
        tc_fence_after();
        // The two pipelines take turns at the exponentials (pipeline 0 first): while one computes
        // its P, the other waits on its MMAs, so neither shares the issue slots and the
        // special-function unit with the other's exponentials.
        if (pipe == 1 || n_exp > 0) {
          if (!tc::mbar_try(smem_addr(turn_mine), (uint32_t)((pipe == 0 ? n_exp - 1 : n_exp) & 1)) &&
              !turn_wait(smem_addr(turn_mine), (uint32_t)((pipe == 0 ? n_exp - 1 : n_exp) & 1),
                         &pipe_done[1 - pipe]))
            ok = false;
        }
        // P = 2^(S·scale - m): scale and offset as packed f32x2 FMAs, the row sum as packed adds
        const uint64_t sc2 = pack_f2(p.scale_log2, p.scale_log2), nm2 = pack_f2(-m_use, -m_use);
        uint64_t acc2[2] = {0ull, 0ull};
#pragma unroll
        for (int c2 = 0; c2 < kKeys; c2 += 32) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float x0, x1;
            unpack_f2(ffma2(pack_u2(r[c2 + 2 * i], r[c2 + 2 * i + 1]), sc2, nm2), x0, x1);
            const float p0 = ex2(x0), p1 = ex2(x1);
            acc2[i & 1] = fadd2(acc2[i & 1], pack_f2(p0, p1));
            __nv_bfloat162 bp = __floats2bfloat162_rn(p0, p1);
            w[i] = *reinterpret_cast<uint32_t*>(&bp);
          }
          tmem_st16(tP + (uint32_t)(c2 / 2), w);
        }
        float s0, s1, s2, s3;
        unpack_f2(acc2[0], s0, s1);
        unpack_f2(acc2[1], s2, s3);
        const float rs = (s0 + s1) + (s2 + s3);
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(turn_other));
        ++n_exp;
        // O rescale after P is written (S registers are dead by then)
        if (__any_sync(0xffffffffu, rescale)) {   // whole warp: tcgen05.ld / st are warp-wide
          uint32_t o[32];
#pragma unroll
          for (int c2 = 0; c2 < kD; c2 += 32) {
            tmem_ld32(tO + (uint32_t)c2, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + (uint32_t)c2, o);
          }
          l *= alpha;
        }
        l += rs;
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(p_full));
      }
      // final O of the tile: after its last PV
      if (!mbar_wait(smem_addr(o_full), (uint32_t)((g - 1) & 1))) ok = false;
      tc_fence_after();
      uint32_t o[kD];
      tmem_ld32(tO, o);
      tmem_ld32(tO + 32, o + 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(o_free));
      // the previous tile's TMA store has finished reading sO before it is rewritten
      if (rl == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      wg_bar(pipe);
      const float inv = __fdividef(1.f, l);
      uint8_t* srow = sO + rl * 128;
#pragma unroll
      for (int v = 0; v < kD / 8; ++v) {
        uint32_t w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          __nv_bfloat162 tt = __floats2bfloat162_rn(__uint_as_float(o[8 * v + 2 * u]) * inv,
                                                    __uint_as_float(o[8 * v + 2 * u + 1]) * inv);
          w[u] = *reinterpret_cast<uint32_t*>(&tt);
        }
        *reinterpret_cast<uint4*>(srow + ((v ^ (rl & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      wg_bar(pipe);
      if (rl == 0 && ok) {   // rows past T are clipped by the tensor map
        tma_store_4d(&to, smem_addr(sO), 0, c.h, c.qb * kRows, c.b);
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      }
    }
    if (lane == 0) pipe_done[pipe] = 1;   // the other pipeline no longer waits for its turn
    if (rl == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // output tiles written
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(*tmem_slot), "r"(512u));
  }
}

// Longest-processing-time-first assignment of the tiles to `pipes`
// pipelines (cost of a tile: 2 per causal key block + 1 for its start and
// output), cached per shape; n = 0 (strided assignment) when the lists do not
// fit the kernel parameter.
static const Sched& schedule(int BH, int n_qblk, int pipes) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int>, std::unique_ptr<Sched>> cache;
  std::lock_guard<std::mutex> g(mu);
  auto key = std::make_tuple(BH, n_qblk, pipes);
  auto it = cache.find(key);
  if (it != cache.end()) return *it->second;
  auto sc = std::make_unique<Sched>();
  sc->n = 0;
  const int64_t n_tiles = (int64_t)BH * n_qblk;
  if (n_tiles + pipes + 1 <= kSchedMax) {
    using Load = std::pair<int64_t, int>;   // (work so far, pipeline), smallest first
    std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
    for (int q = 0; q < pipes; ++q) heap.push({0, q});
    std::vector<std::vector<int>> lists(pipes);
    for (int64_t t = 0; t < n_tiles; ++t) {
      Load l = heap.top();
      heap.pop();
      lists[l.second].push_back((int)t);
      l.first += 2 * (n_qblk - t / BH) + 1;
      heap.push(l);
    }
    int pos = 0;
    for (int q = 0; q < pipes; ++q) {
      sc->v[q] = (uint16_t)pos;
      for (int t : lists[q]) sc->v[pipes + 1 + pos++] = (uint16_t)t;
    }
    sc->v[pipes] = (uint16_t)pos;
    sc->n = pipes + 1 + pos;
  }
  const Sched& ref = *sc;
  cache.emplace(key, std::move(sc));
  return ref;
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
  const int64_t tiles = B * H * p.n_qblk;
  if (tiles > 0x7fffffff) return fail(GPT_ERR_UNSUPPORTED, "attention work too large");
  p.BH = (int)(B * H);
  p.n_tiles = (int)tiles;
  int sms = device_sm_count();
  if (sms <= 0) sms = 148;
  const int64_t pairs = (tiles + kPipes - 1) / kPipes;
  const int grid = (int)(pairs < sms ? pairs : sms);   // persistent: one CTA per SM, two tiles in flight
  const Sched& sc = schedule(p.BH, p.n_qblk, kPipes * grid);
  launch_pdl(attn_tc_kernel, dim3((unsigned)grid), dim3(kThreads), kSmem, st, mq, mk, mv, mo, p, sc);
  return launch_status("attention_tc");
}

}  // namespace attn_tc
}  // namespace gpt
