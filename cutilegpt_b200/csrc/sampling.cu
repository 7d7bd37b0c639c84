// Temperature / top-k / multinomial draw for the last-position logits of a
// decode step, one CTA per sequence, in one launch:
//   cutile_gpt/models/gpt.py:207-225 (logits / temperature, top-k mask
//   `logits < v[:, [-1]]` -> -inf, softmax, torch/cupy multinomial).
//
// 1. threshold: the k-th largest scaled logit, found by a 4-pass radix
//    select (8 bits per pass) over order-preserving 32-bit keys; values equal
//    to the threshold stay in the candidate set, as in the reference mask.
// 2. max and sum of exp over the kept values (fp32).
// 3. inverse CDF: each thread owns a contiguous slice of the row; a block
//    scan of the slice sums finds the slice holding u * sum, whose thread
//    walks it. Summation order is fixed, so a (seed, row, step) triple always
//    draws the same token.
// The uniform u comes from SplitMix64 (Steele, Lea & Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014) applied to (seed, row, step),
// with seed and step read from device memory so the draw can be captured in
// a CUDA graph and replayed step after step.
#include "common.cuh"

namespace gpt {
namespace samp {

constexpr int kThreads = 1024;

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Order-preserving key of a float: larger value -> larger key; NaN -> 0
// (below every number, so it is never kept).
__device__ __forceinline__ uint32_t fkey(float v) {
  if (v != v) return 0u;
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

template <typename T>
__device__ __forceinline__ float ld_scaled(const T* row, int64_t i, float inv_t) {
  return Tr<T>::to_f(row[i]) * inv_t;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) sample_kernel(const T* __restrict__ logits, int64_t ld, int64_t V,
                                                          float inv_t, int64_t top_k,
                                                          const uint64_t* __restrict__ seed_dev,
                                                          const int64_t* __restrict__ step_dev, int64_t step0,
                                                          int64_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t hist[256];
  __shared__ float red[32];
  __shared__ float scan[kThreads / 32];
  __shared__ uint32_t sh_prefix, sh_need;
  __shared__ int64_t sh_pick;
  __shared__ int sh_last;
  const T* row = logits + (int64_t)blockIdx.x * ld;
  const int tid = threadIdx.x;

  // ---- 1. threshold key (k-th largest), or 0 (keep every number)
  uint32_t thr = 0u;
  if (top_k > 0 && top_k < V) {
    uint32_t prefix = 0u, need = (uint32_t)top_k;  // need-th largest among keys matching prefix
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0u;
      __syncthreads();
      const uint32_t hi_mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int64_t i = tid; i < V; i += blockDim.x) {
        const uint32_t k = fkey(ld_scaled(row, i, inv_t));
        if ((k & hi_mask) == (prefix & hi_mask)) atomicAdd(&hist[(k >> shift) & 0xFFu], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        uint32_t acc = 0u;
        int bin = 255;
        for (; bin > 0; --bin) {
          if (acc + hist[bin] >= need) break;
          acc += hist[bin];
        }
        sh_prefix = prefix | ((uint32_t)bin << shift);
        sh_need = need - acc;
      }
      __syncthreads();
      prefix = sh_prefix;
      need = sh_need;
    }
    thr = prefix;
  }

  // ---- 2. max and sum of exp over kept values
  float mx = -INFINITY;
  for (int64_t i = tid; i < V; i += blockDim.x) {
    const float v = ld_scaled(row, i, inv_t);
    if (fkey(v) >= thr && v == v) mx = fmaxf(mx, v);
  }
  mx = warp_max(mx);
  {
    const int w = tid >> 5, lane = tid & 31;
    if (lane == 0) red[w] = mx;
    __syncthreads();
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : -INFINITY;
    mx = warp_max(t);
    __syncthreads();
  }
  if (mx == -INFINITY) {  // nothing finite survives: first index, as an argmax of -inf would give
    if (tid == 0) out[blockIdx.x] = 0;
    return;
  }
  // contiguous slice per thread for the ordered inverse CDF
  const int64_t per = (V + blockDim.x - 1) / blockDim.x;
  const int64_t s0 = (int64_t)tid * per, s1 = min(V, s0 + per);
  float part = 0.f;
  for (int64_t i = s0; i < s1; ++i) {
    const float v = ld_scaled(row, i, inv_t);
    if (fkey(v) >= thr && v == v) part += exp2f((v - mx) * 1.4426950408889634f);
  }
  // exclusive block scan of the slice sums (warp scan + scan of warp totals)
  const int w = tid >> 5, lane = tid & 31;
  float inc = part;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) scan[w] = inc;
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    float t = lane < nw ? scan[lane] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < nw) scan[lane] = t;  // inclusive warp totals
  }
  __syncthreads();
  const float total = scan[(blockDim.x >> 5) - 1];
  const float before = (w > 0 ? scan[w - 1] : 0.f) + inc - part;  // exclusive prefix of this slice

  // ---- 3. draw
  const uint64_t seed = seed_dev ? *seed_dev : 0ull;
  const int64_t step = step0 + (step_dev ? *step_dev : 0);
  const uint64_t r = splitmix64(seed ^ splitmix64((uint64_t)blockIdx.x * 0x632BE59BD9B4E019ull + (uint64_t)step));
  const float u = (float)(r >> 40) * (1.0f / 16777216.0f);  // [0, 1), 24 bits
  const float target = u * total;
  if (tid == 0) {
    sh_pick = INT64_MAX;
    sh_last = -1;
  }
  __syncthreads();
  if (part > 0.f) atomicMax(&sh_last, tid);  // last slice with mass
  __syncthreads();
  // The slice whose [before, before + part) holds the target picks; the last
  // slice with mass also takes a target that rounding left past its end.
  // Competing claims (rounding at a slice edge) resolve to the lowest index.
  const bool mine = part > 0.f && target >= before && (target < before + part || tid == sh_last);
  if (mine) {
    float c = before;
    int64_t pick = -1, last = -1;
    for (int64_t i = s0; i < s1; ++i) {
      const float v = ld_scaled(row, i, inv_t);
      if (fkey(v) >= thr && v == v) {
        const float pv = exp2f((v - mx) * 1.4426950408889634f);
        if (pv > 0.f) last = i;
        c += pv;
        if (c > target && pv > 0.f) { pick = i; break; }
      }
    }
    if (pick < 0) pick = last;
    atomicMin(reinterpret_cast<unsigned long long*>(&sh_pick), (unsigned long long)pick);
  }
  __syncthreads();
  if (tid == 0) out[blockIdx.x] = sh_pick == INT64_MAX ? 0 : sh_pick;
}

}  // namespace samp
}  // namespace gpt

extern "C" {

int gpt_sample(const void* logits, int64_t ld, int64_t B, int64_t V, float temperature, int64_t top_k,
               const uint64_t* seed_dev, const int64_t* step_dev, int64_t step0, int64_t* out, int dtype,
               void* stream) {
  GPT_CHECK_DTYPE(dtype);
  GPT_CHECK_SHAPE(B >= 0 && V > 0 && ld >= V && B < (1LL << 31), "gpt_sample: bad sizes");
  GPT_CHECK_SHAPE(temperature > 0.f && temperature == temperature, "gpt_sample: temperature must be > 0");
  if (B == 0) return GPT_OK;
  GPT_CHECK_ARG(logits && out, "gpt_sample: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const float inv_t = 1.0f / temperature;
  if (dtype == GPT_F32)
    gpt::launch_pdl(gpt::samp::sample_kernel<float>, dim3((unsigned)B), dim3(gpt::samp::kThreads), 0, st,
                    (const float*)logits, ld, V, inv_t, top_k, seed_dev, step_dev, step0, out);
  else
    gpt::launch_pdl(gpt::samp::sample_kernel<__nv_bfloat16>, dim3((unsigned)B), dim3(gpt::samp::kThreads), 0, st,
                    (const __nv_bfloat16*)logits, ld, V, inv_t, top_k, seed_dev, step_dev, step0, out);
  return gpt::launch_status("sample");
}

}  // extern "C"
