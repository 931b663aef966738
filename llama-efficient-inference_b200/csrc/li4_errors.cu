// li4_errors.cu -- per-thread error messages, device queries, version.
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "li4_internal.h"

namespace li4 {

static thread_local char g_last_error[512] = "";

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

void clear_error() { g_last_error[0] = '\0'; }

int check_cuda(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return LI4_OK;
  return set_error(LI4_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

int current_sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= static_cast<int>(cache.size())) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace li4

// 0.2.0: li4_fusion gained the argmax_* fields (a larger struct); the decode program, li4_gather_rows.
extern "C" int li4_version(void) { return (0 << 16) | (2 << 8) | 0; }

extern "C" const char* li4_last_error(void) { return li4::g_last_error; }

extern "C" int li4_debug_set_wait_limits(unsigned allreduce_polls, unsigned program_polls,
                                         unsigned program_wait_extra) {
  int rc = li4::comm_set_wait_limit(allreduce_polls);
  if (rc == LI4_OK) rc = li4::gemv_set_ar_wait_limit(allreduce_polls);
  if (rc == LI4_OK) rc = li4::sample_set_wait_limit(allreduce_polls);
  if (rc == LI4_OK) rc = li4::program_set_wait_limits(program_polls, program_wait_extra);
  if (rc == LI4_OK) li4::clear_error();
  return rc;
}
