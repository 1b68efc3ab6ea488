// Stream-ordered device memory pool (replaces ROCmMemoryManager,
// src/backend/rocm/rocm_memory.cpp:88-205): allocations come from a
// per-device cudaMemPool_t whose release threshold keeps freed memory cached
// for reuse, and frees are ordered on the stream instead of synchronising.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <mutex>
#include <unordered_map>

#include "../../include/pyflame_cuda.h"

namespace pfb {

class CudaMemoryPool {
 public:
  // rocm::ROCmMemoryManager::Config (rocm_memory.hpp:42-50) reduced to what a
  // stream-ordered pool needs.
  struct Config {
    int device = 0;
    size_t release_threshold = 256ull << 20;  // bytes kept cached between calls
    int fail_after_n = 0;                     // fault injection: Nth allocation fails
  };
  explicit CudaMemoryPool(const Config& c);
  ~CudaMemoryPool();
  CudaMemoryPool(const CudaMemoryPool&) = delete;
  CudaMemoryPool& operator=(const CudaMemoryPool&) = delete;

  void* allocate(size_t bytes, cudaStream_t stream);
  // Stream-ordered free; returns cudaFreeAsync's status (destructor paths
  // may ignore it, every other caller checks it).
  cudaError_t deallocate(void* p, cudaStream_t stream);
  pfc_memory_stats stats() const;
  void add_resident(long long delta) { resident_ += delta; }

 private:
  Config cfg_;
  cudaMemPool_t pool_ = nullptr;
  mutable std::mutex mu_;
  std::unordered_map<void*, size_t> sizes_;
  size_t allocated_ = 0, peak_ = 0, n_alloc_ = 0, n_free_ = 0, hits_ = 0, misses_ = 0;
  long long resident_ = 0;
};

}  // namespace pfb
