// Host-side helpers shared by the C-ABI translation units: status codes, the
// thread-local last-error string, and argument / CUDA checks that turn into a
// returned status instead of an abort (the reference raises PanicError through
// RuntimeCheck, python/sglite/kernels/csrc/include/sglite/utils.h:42-92).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <string>

namespace awqb {

enum Status : int {
  kOk = 0,
  kInvalidArgument = 1,  // Python shim raises ValueError
  kUnsupported = 2,      // ValueError (shape/config the kernels do not cover)
  kCudaError = 3,        // RuntimeError
  kNcclError = 4,        // RuntimeError
  kDeviceTimeout = 5,    // RuntimeError: a bounded device wait gave up
};

void set_last_error(const std::string& msg);
const char* get_last_error();

int device_sm_count();  // of the current device, cached per device

}  // namespace awqb

#define AWQB_REQUIRE(cond, code, ...)                        \
  do {                                                       \
    if (!(cond)) {                                           \
      char _buf[512];                                        \
      snprintf(_buf, sizeof(_buf), __VA_ARGS__);             \
      ::awqb::set_last_error(_buf);                          \
      return (code);                                         \
    }                                                        \
  } while (0)

#define AWQB_CUDA(expr)                                                              \
  do {                                                                               \
    cudaError_t _e = (expr);                                                         \
    if (_e != cudaSuccess) {                                                         \
      char _buf[512];                                                                \
      snprintf(_buf, sizeof(_buf), "%s failed: %s (%s:%d)", #expr,                   \
               cudaGetErrorString(_e), __FILE__, __LINE__);                          \
      ::awqb::set_last_error(_buf);                                                  \
      return ::awqb::kCudaError;                                                     \
    }                                                                                \
  } while (0)

#define AWQB_LAUNCH_CHECK() AWQB_CUDA(cudaGetLastError())
