#include "memory_pool.hpp"

#include <algorithm>
#include <string>

#include "common.hpp"

namespace pfb {

CudaMemoryPool::CudaMemoryPool(const Config& c) : cfg_(c) {
  cudaMemPoolProps props = {};
  props.allocType = cudaMemAllocationTypePinned;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = c.device;
  PFB_CUDA(cudaMemPoolCreate(&pool_, &props));
  uint64_t thr = c.release_threshold;
  PFB_CUDA(cudaMemPoolSetAttribute(pool_, cudaMemPoolAttrReleaseThreshold, &thr));
}

CudaMemoryPool::~CudaMemoryPool() {
  if (pool_) cudaMemPoolDestroy(pool_);
}

void* CudaMemoryPool::allocate(size_t bytes, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(mu_);
  bytes = std::max<size_t>(bytes, 256);
  if (cfg_.fail_after_n > 0 && (int)(n_alloc_ + 1) >= cfg_.fail_after_n)
    fail(PFC_ERR_OUT_OF_MEMORY, "injected allocation failure (allocation " + std::to_string(n_alloc_ + 1) + ")");
  uint64_t reserved_before = 0, reserved_after = 0;
  cudaMemPoolGetAttribute(pool_, cudaMemPoolAttrReservedMemCurrent, &reserved_before);
  void* p = nullptr;
  cudaError_t e = cudaMallocFromPoolAsync(&p, bytes, pool_, stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(e == cudaErrorMemoryAllocation ? PFC_ERR_OUT_OF_MEMORY : PFC_ERR_CUDA,
         "device allocation of " + std::to_string(bytes) + " bytes failed: " + cudaGetErrorString(e));
  }
  cudaMemPoolGetAttribute(pool_, cudaMemPoolAttrReservedMemCurrent, &reserved_after);
  if (reserved_after > reserved_before) ++misses_;
  else ++hits_;
  sizes_[p] = bytes;
  allocated_ += bytes;
  peak_ = std::max(peak_, allocated_);
  ++n_alloc_;
  return p;
}

cudaError_t CudaMemoryPool::deallocate(void* p, cudaStream_t stream) {
  if (!p) return cudaSuccess;
  std::lock_guard<std::mutex> lock(mu_);
  auto it = sizes_.find(p);
  if (it == sizes_.end()) return cudaSuccess;
  allocated_ -= it->second;
  sizes_.erase(it);
  ++n_free_;
  return cudaFreeAsync(p, stream);
}

pfc_memory_stats CudaMemoryPool::stats() const {
  std::lock_guard<std::mutex> lock(mu_);
  pfc_memory_stats s = {};
  s.total_allocated = allocated_;
  s.peak_allocated = peak_;
  s.total_allocations = n_alloc_;
  s.total_deallocations = n_free_;
  s.cache_hits = hits_;
  s.cache_misses = misses_;
  s.resident_constant_bytes = (size_t)std::max<long long>(0, resident_);
  return s;
}

}  // namespace pfb
