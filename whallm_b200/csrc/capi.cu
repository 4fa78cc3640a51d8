// Error state and small device queries shared by every entry point.
#include <mutex>
#include <string>

#include "wm_common.cuh"

namespace wm {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string &msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }

int sm_count() {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace wm

extern "C" {

const char *w_last_error(void) { return wm::g_last_error.c_str(); }

int w_abi_version(void) { return 1; }

}  // extern "C"
