// Self-check of the failure path the tensor-core kernels share: an mbarrier
// wait bounded by the global timer that gives up, records PFC_ERR_TIMEOUT in
// the device error flag and lets the kernel return, so the host sees an error
// status and the context stays usable.  The kernel here waits on a barrier
// that nothing arrives on, through the same wait helper as the GEMM and
// attention kernels, with a caller-chosen limit.  Nothing faults or hangs.
#include <cuda_runtime.h>

#include "../common.hpp"
#include "kernels.hpp"
#include "tcgen05.cuh"

namespace pfb {
namespace {

__global__ void wait_check_kernel(int* err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // no thread ever arrives: the phase cannot complete, the wait must give up
  if (threadIdx.x == 0) (void)mbar_wait_for(smem_u32(&bar), 0u, err, limit_ns);
}

}  // namespace

void launch_wait_check(int* err, int64_t limit_us, cudaStream_t stream) {
  PFB_CHECK_ARG(err, "wait check: null error flag");
  PFB_CHECK_ARG(limit_us > 0 && limit_us <= 5000000, "wait check: limit must be in (0, 5 s]");
  wait_check_kernel<<<1, 32, 0, stream>>>(err, (unsigned long long)limit_us * 1000ull);
  PFB_CUDA(cudaGetLastError());
}

}  // namespace pfb
