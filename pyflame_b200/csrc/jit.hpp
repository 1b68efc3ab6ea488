// NVRTC compilation of generated kernels to sm_100a cubins, loaded through
// the CUDA runtime's library API (no libcuda link-time dependency).
#pragma once

#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <unordered_map>

namespace pfb {

class JitCache {
 public:
  // Compile (once per distinct source) and return the kernel handle on the
  // current device.  `key` identifies the source; `name` is the extern "C"
  // kernel symbol.
  cudaKernel_t get(const std::string& key, const std::string& source, const std::string& name);
  // Compile only (no device needed): returns the cubin size.  Used to check
  // generated code on hosts without a GPU.
  static size_t compile_only(const std::string& source, std::string* log);
  size_t modules() const { return libs_.size(); }

 private:
  struct Entry {
    std::string cubin;
    std::unordered_map<int, cudaLibrary_t> lib_by_device;
  };
  std::mutex mu_;
  std::unordered_map<std::string, Entry> libs_;
};

JitCache& global_jit();
std::string hash_hex(const std::string& s);

}  // namespace pfb
