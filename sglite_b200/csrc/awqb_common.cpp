// Status / last-error plumbing shared by every C-ABI entry point.
#include "awqb_common.h"

#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "awqb200.h"

namespace awqb {

namespace {
thread_local std::string t_last_error;
}

void set_last_error(const std::string& msg) { t_last_error = msg; }
const char* get_last_error() { return t_last_error.c_str(); }

int device_sm_count() {
  static int counts[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if (counts[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

}  // namespace awqb

extern "C" const char* awqb_last_error(void) { return awqb::get_last_error(); }

extern "C" int awqb_abi_version(void) { return AWQB_ABI_VERSION; }
