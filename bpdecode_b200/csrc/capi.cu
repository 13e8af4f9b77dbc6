// Library-wide C ABI helpers: version string and per-thread error messages.
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

}  // namespace bpd

extern "C" const char* bpd_version(void) { return "bpdecode_b200 0.1.0 (sm_100a)"; }

extern "C" const char* bpd_last_error(void) { return bpd::g_last_error; }
