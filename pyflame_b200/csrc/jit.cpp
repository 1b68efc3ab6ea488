#include "jit.hpp"

#include <nvrtc.h>

#include <cstdio>
#include <vector>

#include "common.hpp"

namespace pfb {

std::string hash_hex(const std::string& s) {
  // FNV-1a 64 twice with different offsets -> 128-bit hex key.
  uint64_t h1 = 0xcbf29ce484222325ULL, h2 = 0x84222325cbf29ce4ULL;
  for (unsigned char c : s) {
    h1 = (h1 ^ c) * 0x100000001b3ULL;
    h2 = (h2 ^ c) * 0x100000001b3ULL + 0x9e37;
  }
  char buf[40];
  std::snprintf(buf, sizeof buf, "%016llx%016llx", (unsigned long long)h1, (unsigned long long)h2);
  return buf;
}

static std::string nvrtc_compile(const std::string& source, std::string* log_out) {
  nvrtcProgram prog;
  if (nvrtcCreateProgram(&prog, source.c_str(), "pyflame_jit.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
    fail(PFC_ERR_JIT, "nvrtcCreateProgram failed");
  // --fmad=false keeps every IR operation separately rounded (the CPU
  // reference evaluates a*b and +c as two float operations).
  const char* opts[] = {"--gpu-architecture=sm_100a", "--std=c++17", "--fmad=false",
                        "-default-device", "-lineinfo"};
  nvrtcResult r = nvrtcCompileProgram(prog, 5, opts);
  size_t log_size = 0;
  nvrtcGetProgramLogSize(prog, &log_size);
  std::string log(log_size, '\0');
  if (log_size) nvrtcGetProgramLog(prog, log.data());
  if (log_out) *log_out = log;
  if (r != NVRTC_SUCCESS) {
    nvrtcDestroyProgram(&prog);
    fail(PFC_ERR_JIT, std::string("NVRTC compile failed: ") + nvrtcGetErrorString(r) + "\n" + log +
                          "\n--- source ---\n" + source);
  }
  size_t n = 0;
  nvrtcGetCUBINSize(prog, &n);
  std::string cubin(n, '\0');
  nvrtcGetCUBIN(prog, cubin.data());
  nvrtcDestroyProgram(&prog);
  return cubin;
}

size_t JitCache::compile_only(const std::string& source, std::string* log) {
  return nvrtc_compile(source, log).size();
}

cudaKernel_t JitCache::get(const std::string& key, const std::string& source, const std::string& name) {
  std::lock_guard<std::mutex> lock(mu_);
  Entry& e = libs_[key];
  if (e.cubin.empty()) e.cubin = nvrtc_compile(source, nullptr);
  int dev = 0;
  PFB_CUDA(cudaGetDevice(&dev));
  auto it = e.lib_by_device.find(dev);
  cudaLibrary_t lib;
  if (it == e.lib_by_device.end()) {
    PFB_CUDA(cudaLibraryLoadData(&lib, e.cubin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0));
    e.lib_by_device[dev] = lib;
  } else {
    lib = it->second;
  }
  cudaKernel_t k;
  PFB_CUDA(cudaLibraryGetKernel(&k, lib, name.c_str()));
  return k;
}

JitCache& global_jit() {
  static JitCache* c = new JitCache();  // lives until exit
  return *c;
}

}  // namespace pfb
