// Library-level C entry points: version, thread-local error string, device
// error word, SM count.
#include <stdarg.h>
#include <mutex>

#include "common.cuh"

namespace gpt {

static thread_local std::string t_last_error;
static thread_local int64_t t_launches = 0;
static thread_local cudaError_t t_launch_error = cudaSuccess;

void note_launch_error(cudaError_t e) { t_launch_error = e; }

void set_error(const std::string& msg) { t_last_error = msg; }

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return status;
}

int launch_status(const char* what) {
  ++t_launches;
  cudaError_t e = t_launch_error;
  t_launch_error = cudaSuccess;
  cudaError_t last = cudaGetLastError();
  if (e == cudaSuccess) e = last;
  if (e != cudaSuccess)
    return fail(GPT_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return GPT_OK;
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  // One cached value per device ordinal (B200 nodes have at most 8-16).
  static int cache[64] = {0};
  static std::mutex mu;
  if (dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> g(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace gpt

extern "C" {

int gpt_set_wait_limit_ns(uint64_t ns) {
  GPT_CHECK_ARG(ns > 0, "gpt_set_wait_limit_ns: the limit must be positive");
  unsigned long long v = (unsigned long long)ns;
  cudaError_t e = cudaMemcpyToSymbol(gpt::g_wait_limit_ns, &v, sizeof(v));
  if (e != cudaSuccess) return gpt::fail(GPT_ERR_CUDA, "gpt_set_wait_limit_ns: %s", cudaGetErrorString(e));
  return GPT_OK;
}



int gpt_version(void) { return 1; }

const char* gpt_last_error_string(void) { return gpt::t_last_error.c_str(); }

int gpt_sm_count(void) { return gpt::device_sm_count(); }

int64_t gpt_launch_count(void) { return gpt::t_launches; }

int gpt_device_error(int* code_out) {
  GPT_CHECK_ARG(code_out != nullptr, "gpt_device_error: null code_out");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess)
    return gpt::fail(GPT_ERR_CUDA, "gpt_device_error: %s", cudaGetErrorString(e));
  unsigned int v = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&v, gpt::g_dev_error, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(gpt::g_dev_error, &zero, sizeof(zero));
  if (e != cudaSuccess)
    return gpt::fail(GPT_ERR_CUDA, "gpt_device_error: %s", cudaGetErrorString(e));
  *code_out = (int)v;
  if (v & GPT_DEVERR_TIMEOUT) return gpt::fail(GPT_ERR_TIMEOUT, "a bounded device wait timed out");
  if (v & GPT_DEVERR_INDEX) return gpt::fail(GPT_ERR_SHAPE, "a kernel saw an out-of-range index");
  return GPT_OK;
}

}  // extern "C"
