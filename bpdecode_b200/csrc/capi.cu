// Library-wide C ABI helpers: version string and per-thread error messages.
#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace bpd {

namespace {
thread_local char g_last_error[512] = "";
}

bpd_status fail(bpd_status code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

bpd_status check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(BPD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return BPD_OK;
}

int32_t sm_count() {
  static std::atomic<int32_t> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int32_t n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    n = v;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

}  // namespace bpd

extern "C" const char* bpd_version(void) { return "bpdecode_b200 0.1.0 (sm_100a)"; }

extern "C" const char* bpd_last_error(void) { return bpd::g_last_error; }
