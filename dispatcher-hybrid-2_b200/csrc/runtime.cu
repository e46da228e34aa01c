// Error reporting, device queries and small helpers shared by all entry points.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>

#include "common.cuh"

namespace dh {

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(DH_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return DH_OK;
}

// process-wide; negative = the default limit
static std::atomic<long long> g_wait_limit{-1};

uint32_t wait_limit() {
  const long long v = g_wait_limit.load(std::memory_order_relaxed);
  if (v < 0) return kDefaultWaitLimit;
  return v > 0xffffffffll ? 0xffffffffu : (uint32_t)v;
}

int sm_count() {
  static thread_local int cached_dev = -1, cached = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev != cached_dev) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached = n;
    cached_dev = dev;
  }
  return cached;
}

}  // namespace dh

extern "C" const char* dh_version(void) { return "dispatcher_b200 0.1 (sm_100a)"; }

extern "C" const char* dh_last_error(void) { return dh::g_err; }

extern "C" int dh_sm_count(int* out) {
  if (!out) return dh::set_error(DH_ERR_ARG, "dh_sm_count: null output");
  *out = dh::sm_count();
  return DH_OK;
}

extern "C" int dh_set_wait_limit(long long polls) {
  dh::g_wait_limit.store(polls < 0 ? -1 : polls, std::memory_order_relaxed);
  return DH_OK;
}
