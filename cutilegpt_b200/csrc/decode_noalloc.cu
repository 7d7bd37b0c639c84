// gpt_attention_decode_noalloc: the split-KV decode attention for callers
// that cannot allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits — a host
// runtime whose memory is owned by a fixed arena or a foreign allocator it
// must not bypass, a plugin loaded into a process that forbids allocation
// after start-up (allocation can synchronise the device and break latency
// guarantees), or a real-time loop that must never block on the driver's
// allocator. Those callers can still pass inputs and outputs they own, but
// not the workspace gpt_attention_decode wants for its per-split partials.
//
// Here the partials live in a fixed device array of this library,
// kNoAllocScratchBytes (256 KiB) per GPU, allocated when the library is
// loaded and held until the process exits. Requests needing more are
// rejected with GPT_ERR_SHAPE. Every call on a device shares the array: two
// calls whose kernels overlap on the GPU (different streams, no ordering)
// race on it. Each split writes all of its partial values before the
// combine step reads them, so nothing has to be cleared between calls; the
// previous call's contents are simply overwritten.
#include <mutex>

#include "common.cuh"

namespace gpt {
namespace noalloc {

constexpr int64_t kNoAllocScratchBytes = GPT_NOALLOC_DECODE_SCRATCH_BYTES;
static_assert(kNoAllocScratchBytes % 256 == 0, "scratch size must keep 256-byte alignment");

// Device-resident scratch. In host code this name is only a stand-in for
// the symbol, not a device address; the address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) float g_decode_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of g_decode_scratch on the current device, looked up once
// per device (with that device current) and cached for the life of the
// process. The cache does not survive cudaDeviceReset() (or any other reset
// of the device's primary context): the module is then loaded again and the
// array may move, so a process that resets a device must not call this entry
// point on it afterwards.
static int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(GPT_ERR_CUDA, "gpt_attention_decode_noalloc: %s", cudaGetErrorString(e));
  static void* cache[64] = {nullptr};
  static std::mutex mu;
  if (dev < 0 || dev >= 64) return fail(GPT_ERR_UNSUPPORTED, "gpt_attention_decode_noalloc: device %d", dev);
  std::lock_guard<std::mutex> g(mu);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(GPT_ERR_CUDA, "gpt_attention_decode_noalloc: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
    cache[dev] = p;
  }
  *out = cache[dev];
  return GPT_OK;
}

}  // namespace noalloc
}  // namespace gpt

extern "C" int gpt_attention_decode_noalloc(const void* q, int64_t ld_q, const void* k_cache,
                                            const void* v_cache, void* out, int64_t ld_out, int64_t B,
                                            int64_t H, int64_t D, int64_t Tmax, int64_t L,
                                            const int64_t* len_dev, float scale, int dtype, void* stream) {
  const int64_t need = gpt_attention_decode_workspace_size(B, H, D, len_dev ? Tmax : L);
  if (need > gpt::noalloc::kNoAllocScratchBytes)
    return gpt::fail(GPT_ERR_SHAPE,
                     "gpt_attention_decode_noalloc: these sizes need %lld bytes of split-KV scratch, more "
                     "than the library's fixed %lld-byte array; use gpt_attention_decode with a workspace",
                     (long long)need, (long long)gpt::noalloc::kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (need > 0) {
    int s = gpt::noalloc::scratch_address(&scratch);
    if (s != GPT_OK) return s;
  }
  return gpt_attention_decode(q, ld_q, k_cache, v_cache, out, ld_out, B, H, D, Tmax, L, len_dev, scale,
                              scratch, dtype, stream);
}
