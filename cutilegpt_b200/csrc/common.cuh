// Shared helpers for libgpt_b200: status plumbing, dtype traits, device
// error word, small math. Included once by libgpt_b200.cu, the single
// translation unit of the library.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <string>
#include <utility>

#include "../../include/gpt_b200.h"

namespace gpt {

// ---- host-side error reporting (thread-local last error) -------------------
void set_error(const std::string& msg);
int fail(int status, const char* fmt, ...);

#define GPT_CHECK_ARG(cond, ...)                                   \
  do {                                                             \
    if (!(cond)) return ::gpt::fail(GPT_ERR_ARG, __VA_ARGS__);     \
  } while (0)
#define GPT_CHECK_SHAPE(cond, ...)                                 \
  do {                                                             \
    if (!(cond)) return ::gpt::fail(GPT_ERR_SHAPE, __VA_ARGS__);   \
  } while (0)
#define GPT_CHECK_ALIGN(cond, ...)                                 \
  do {                                                             \
    if (!(cond)) return ::gpt::fail(GPT_ERR_ALIGN, __VA_ARGS__);   \
  } while (0)
#define GPT_CHECK_DTYPE(dt)                                                     \
  do {                                                                          \
    if ((dt) != GPT_F32 && (dt) != GPT_BF16)                                    \
      return ::gpt::fail(GPT_ERR_DTYPE, "unsupported dtype %d", (int)(dt));     \
  } while (0)

// Checks the launch that was just issued; returns GPT_OK or GPT_ERR_CUDA.
int launch_status(const char* what);
// Records a launch error returned by cudaLaunchKernelEx for launch_status().
void note_launch_error(cudaError_t e);

// Programmatic dependent launch: every kernel of this library is launched
// with programmatic stream serialisation, so its CTAs may start (set up
// barriers, TMEM, prefetch weights) while the previous kernel in the stream
// is still running. Each kernel calls pdl_wait() before it reads anything a
// predecessor may write or writes anything a predecessor may read, and
// pdl_trigger() once its own CTAs no longer need to hold back the next
// kernel. The next kernel's CTAs start only after every CTA of this grid has
// started, so early triggering cannot starve this grid's later waves.
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) note_launch_error(e);
}

// Same, for a kernel launched in thread-block clusters of `cluster_x` CTAs.
template <typename... KArgs, typename... Args>
inline void launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                               unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) note_launch_error(e);
}

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

int device_sm_count();

// ---- device error word ----------------------------------------------------
// Bounded waits and index checks record a code here instead of trapping.
// Host reads and clears it with gpt_device_error(). The library is one
// translation unit (libgpt_b200.cu includes every kernel file), so this is
// a single device symbol.
#define GPT_DEVERR_TIMEOUT 0x1u
#define GPT_DEVERR_INDEX 0x2u
__device__ unsigned int g_dev_error;
__device__ __forceinline__ void record_device_error(unsigned int code) {
  atomicOr(&g_dev_error, code);
}
// Limit of every bounded wait (mbarrier phase waits of the tensor-core
// kernels), in ns of %globaltimer. 4 s by default; gpt_set_wait_limit_ns()
// changes it for the current device (tests shorten it to make a wait run out).
__device__ unsigned long long g_wait_limit_ns = 4000000000ull;

// ---- dtype traits ----------------------------------------------------------
template <typename T> struct Tr;
template <> struct Tr<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Tr<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// tanh-GELU of GPT-2 (cutile_gpt/kernels/gelu.py:16-17, :36-38):
// 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))). tanh is CUDA's tanhf
// (accurate to a few ulp) for fp32 work; the bf16 path uses the hardware
// tanh.approx.f32 instruction (max rel. error ~2^-11, far below bf16's 2^-8).
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
template <bool kFast>
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  float inner = k0 * fmaf(k1 * x, x * x, x);
  float t = kFast ? tanh_fast(inner) : tanhf(inner);
  return 0.5f * x * (1.0f + t);
}

// Two tanh-GELUs with one packed tanh: the tanh arguments are rounded to
// f16 and go through tanh.approx.f16x2 (two results per MUFU issue, max rel.
// error ~2^-10.7, still below the bf16 output's 2^-8). The GELU epilogue of
// a large GEMM is bound by MUFU throughput (16 results per clock per SM),
// so halving the MUFU issues halves its cost.
__device__ __forceinline__ void gelu_tanh2_fast(float& x0, float& x1) {
  const float k0 = 0.7978845608028654f;             // sqrt(2/pi)
  const float k01 = 0.7978845608028654f * 0.044715f;
  const float u0 = x0 * fmaf(k01, x0 * x0, k0);
  const float u1 = x1 * fmaf(k01, x1 * x1, k0);
  uint32_t h, t;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(u1), "f"(u0));
  asm("tanh.approx.f16x2 %0, %1;" : "=r"(t) : "r"(h));
  float t0, t1;
  asm("{\n .reg .f16 lo, hi;\n mov.b32 {lo, hi}, %2;\n cvt.f32.f16 %0, lo;\n cvt.f32.f16 %1, hi;\n}"
      : "=f"(t0), "=f"(t1) : "r"(t));
  const float h0 = 0.5f * x0, h1 = 0.5f * x1;
  x0 = fmaf(h0, t0, h0);
  x1 = fmaf(h1, t1, h1);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

}  // namespace gpt

