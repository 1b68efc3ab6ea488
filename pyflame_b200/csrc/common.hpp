// Shared helpers: error type carrying a C-ABI status code, CUDA checks.
#pragma once

#include <cstdint>
#include <cstdio>
#include <mutex>
#include <stdexcept>
#include <string>

#include <cuda_runtime.h>

#include "../../include/pyflame_cuda.h"

namespace pfb {

// Exception used inside the library; the C-ABI layer turns it into a status
// code (no exception crosses extern "C", like rocm_kernels.hip:740-806).
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& msg) : std::runtime_error(msg), code(c) {}
};

[[noreturn]] inline void fail(int code, const std::string& msg) { throw Error(code, msg); }

#define PFB_CHECK_ARG(cond, msg)                                               \
  do {                                                                         \
    if (!(cond)) ::pfb::fail(PFC_ERR_INVALID_ARGUMENT, std::string(msg));      \
  } while (0)

#define PFB_CUDA(expr)                                                         \
  do {                                                                         \
    cudaError_t _e = (expr);                                                   \
    if (_e != cudaSuccess) {                                                   \
      ::pfb::fail(_e == cudaErrorMemoryAllocation ? PFC_ERR_OUT_OF_MEMORY      \
                                                  : PFC_ERR_CUDA,              \
                  std::string(#expr) + ": " + cudaGetErrorString(_e));         \
    }                                                                          \
  } while (0)

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

void set_last_error(const std::string& msg);

// The calling thread's current device, checked (kernel set-up caches are
// indexed by it and hold 64 devices).
inline int current_device() {
  int dev = 0;
  PFB_CUDA(cudaGetDevice(&dev));
  PFB_CHECK_ARG(dev >= 0 && dev < 64, "device index above 63");
  return dev;
}

// Multiprocessor count of `dev`, queried once per device under std::call_once,
// so host threads launching at the same time never read a half-written entry.
inline int device_sm_count(int dev) {
  static std::once_flag once[64];
  static int sms[64];
  std::call_once(once[dev & 63], [dev] {
    int v = 0;
    PFB_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
    sms[dev & 63] = v > 0 ? v : 148;
  });
  return sms[dev & 63];
}

}  // namespace pfb
