// Error reporting and version entry points of the C ABI.
#include <stdarg.h>

#include <atomic>

#include "gs_common.cuh"

namespace gs {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_last_error[0] = '\0'; }

static std::atomic<unsigned long long> g_launches{0};

void note_launches(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

}  // namespace gs

extern "C" {

int gs_version(void) { return 100; }  // 0.1.0

const char* gs_last_error(void) { return gs::g_last_error; }

uint64_t gs_kernel_launch_count(void) { return gs::g_launches.load(std::memory_order_relaxed); }

int gs_set_wait_limit(int polls) {
  gs::clear_error();
  if (polls < 0) return gs::set_error(GS_ERR_INVALID_ARG, "polls must be >= 0");
  int e = gs::binning_set_wait_limit(polls);
  if (e != 0) return gs::set_error(GS_ERR_CUDA, "gs_set_wait_limit: %s", cudaGetErrorString((cudaError_t)e));
  return GS_OK;
}

int gs_wait_failures(uint64_t* count, int reset) {
  gs::clear_error();
  if (!count) return gs::set_error(GS_ERR_INVALID_ARG, "count is NULL");
  unsigned long long a = 0, b = 0;
  int e = gs::binning_wait_failures(&a, reset);
  if (e == 0) e = gs::preprocess_wait_failures(&b, reset);
  if (e != 0)
    return gs::set_error(GS_ERR_CUDA, "gs_wait_failures: %s", cudaGetErrorString((cudaError_t)e));
  *count = a + b;
  return GS_OK;
}

}  // extern "C"
