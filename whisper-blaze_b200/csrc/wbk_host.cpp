// Host-side error plumbing and device queries shared by every libwbk entry point.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "wbk.h"

namespace wbk {

namespace {
thread_local std::string g_last_error;
std::atomic<uint64_t> g_wait_timeout_ns{0};  // wbk_set_wait_timeout_ns; 0 = default
}

uint64_t wait_timeout_override_ns() { return g_wait_timeout_ns.load(std::memory_order_relaxed); }

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return WBK_OK;
  return fail(WBK_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  const int dev = current_device();
  if (dev < 0) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace wbk

extern "C" {

int wbk_version(void) { return 1 * 10000 + 0 * 100 + 0; }

const char* wbk_last_error(void) { return wbk::g_last_error.c_str(); }

int wbk_set_wait_timeout_ns(uint64_t timeout_ns) {
  if (timeout_ns > 60ull * 1000000000ull)
    return wbk::fail(WBK_ERR_INVALID_ARG, "wbk_set_wait_timeout_ns: %llu ns is above the 60 s limit",
                     static_cast<unsigned long long>(timeout_ns));
  wbk::g_wait_timeout_ns.store(timeout_ns, std::memory_order_relaxed);
  return WBK_OK;
}

}  // extern "C"
