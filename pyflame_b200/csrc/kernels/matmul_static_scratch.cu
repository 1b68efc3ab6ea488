// matmul_static_scratch.cu — fp32 matmul for callers that cannot allocate
// device memory.
//
// pfk_matmul_tf32x3_static computes C = A @ B (A [M,K], B [K,N], C [M,N],
// all fp32 dense row-major) with the
// same 3xTF32 tcgen05 GEMM and operand split as pfk_split_tf32 + pfk_gemm.
// Those entry points need the caller to supply device buffers for the split
// operands and the error flag; this one takes them from a fixed scratch array
// compiled into this file, so a call performs no device allocation at all.
//
// Who needs it: a host that has already handed every byte of device memory
// to its own allocator (a serving runtime's arena, a framework's caching
// allocator) and cannot grant a library more, and latency-critical paths on
// which cudaMalloc/cudaFree would block or synchronise the device.
//
// Limits and rules:
//  - The operands' split copies must fit the scratch array: with
//    Kp = K rounded up to 32, the call needs
//    256 + 2*ru(4*M*Kp) + 2*ru(4*N*Kp) bytes (ru = round up to 256), at most
//    kScratchBytes (64 MiB); e.g. M = N = K = 1536 fits, M = N = K = 2048
//    does not.  Larger problems are rejected with PFC_ERR_INVALID_ARGUMENT
//    and nothing is launched.
//  - Every call in the process shares the one array (one copy per device),
//    so calls that overlap in time race on it: serialise them, for example
//    by issuing them on one stream.
//  - The array holds 64 MiB on every device where this library's device
//    code is loaded (with CUDA_MODULE_LOADING=EAGER: at context creation),
//    called or not.
//  - The first call on a device looks the array's device address up
//    (cudaGetSymbolAddress, which may load this file's device code into the
//    context).  Make that first call before any stream capture begins.
#include <cstdint>
#include <mutex>
#include <string>

#include <cuda_runtime.h>

#include "../common.hpp"
#include "kernels.hpp"

namespace {

constexpr size_t kScratchBytes = size_t(64) << 20;
constexpr size_t kFlagBytes = 256;  // the wait-timeout flag, then the operands
constexpr int kMaxDevices = 64;

// The only storage this entry point uses.  Host code never takes this name as
// a device address; scratch_base() asks the runtime for it per device.
static __device__ __align__(256) unsigned char g_matmul_scratch[kScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_base[kMaxDevices] = {};

size_t ru256(size_t b) { return (b + 255) / 256 * 256; }

// Device address of g_matmul_scratch on the current device (set up once).
unsigned char* scratch_base() {
  int dev = -1;
  PFB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) pfb::fail(PFC_ERR_NO_DEVICE, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_scratch_base[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_matmul_scratch);
    if (e != cudaSuccess || !p)
      pfb::fail(PFC_ERR_CUDA, std::string("scratch set-up: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    g_scratch_base[dev] = p;
  }
  return static_cast<unsigned char*>(g_scratch_base[dev]);
}

}  // namespace

extern "C" PFC_API int pfk_matmul_tf32x3_static(const float* a, const float* b, float* c, int64_t M, int64_t N,
                                                int64_t K, int* err, void* stream) {
  try {
    PFB_CHECK_ARG(M > 0 && N > 0 && K > 0, "pfk_matmul_tf32x3_static: M, N and K must be positive");
    PFB_CHECK_ARG(M < (int64_t(1) << 31) && N < (int64_t(1) << 31) && K < (int64_t(1) << 31),
                  "pfk_matmul_tf32x3_static: dimension too large");
    const int64_t kpad = pfb::round_up(K, 32);
    const size_t a_bytes = ru256(size_t(M) * size_t(kpad) * 4), b_bytes = ru256(size_t(N) * size_t(kpad) * 4);
    const size_t need = kFlagBytes + 2 * a_bytes + 2 * b_bytes;
    if (need > kScratchBytes)
      pfb::fail(PFC_ERR_INVALID_ARGUMENT, "pfk_matmul_tf32x3_static: M=" + std::to_string(M) + " N=" +
                                              std::to_string(N) + " K=" + std::to_string(K) + " needs " +
                                              std::to_string(need) + " bytes of scratch; the maximum is " +
                                              std::to_string(kScratchBytes));
    PFB_CHECK_ARG(a && b && c, "pfk_matmul_tf32x3_static: null pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned char* base = scratch_base();
    int* flag = reinterpret_cast<int*>(base);
    float* a_hi = reinterpret_cast<float*>(base + kFlagBytes);
    float* a_lo = reinterpret_cast<float*>(base + kFlagBytes + a_bytes);
    float* b_hi = reinterpret_cast<float*>(base + kFlagBytes + 2 * a_bytes);
    float* b_lo = reinterpret_cast<float*>(base + kFlagBytes + 2 * a_bytes + b_bytes);

    // The flag must start at zero; the split kernels write every operand
    // element, K padding included, so nothing else needs clearing.
    PFB_CUDA(cudaMemsetAsync(flag, 0, sizeof(int), s));

    pfb::PrepLaunch pa;  // A [M,K] row-major: rows M, K contiguous
    pa.src = a;
    pa.rank = 2;
    pa.shape[0] = M; pa.shape[1] = K;
    pa.stride[0] = K; pa.stride[1] = 1;
    pa.precision = PFC_PRECISION_TF32X3;
    pa.hi = a_hi; pa.lo = a_lo; pa.kpad = kpad;
    pfb::launch_prepare(pa, s);

    pfb::PrepLaunch pb;  // B [K,N] row-major read as N rows of K (stride N along K)
    pb.src = b;
    pb.rank = 2;
    pb.shape[0] = N; pb.shape[1] = K;
    pb.stride[0] = 1; pb.stride[1] = N;
    pb.precision = PFC_PRECISION_TF32X3;
    pb.hi = b_hi; pb.lo = b_lo; pb.kpad = kpad;
    pfb::launch_prepare(pb, s);

    pfb::GemmLaunch g;
    g.precision = PFC_PRECISION_TF32X3;
    g.a_hi = a_hi; g.a_lo = a_lo; g.b_hi = b_hi; g.b_lo = b_lo;
    g.batch = 1; g.M = M; g.N = N; g.K = K; g.kpad = kpad;
    g.c = c; g.c_sm = N; g.c_sn = 1;
    g.err = flag;
    pfb::launch_gemm(g, s);

    if (err) PFB_CUDA(cudaMemcpyAsync(err, flag, sizeof(int), cudaMemcpyDeviceToDevice, s));
    return PFC_OK;
  } catch (const pfb::Error& e) {
    pfb::set_last_error(e.what());
    return e.code;
  } catch (const std::exception& e) {
    pfb::set_last_error(e.what());
    return PFC_ERR_INTERNAL;
  } catch (...) {
    pfb::set_last_error("unknown error");
    return PFC_ERR_INTERNAL;
  }
}
