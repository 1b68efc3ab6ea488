// Tensor-core GEMM for sm_100a: C[b,m,n] = epilogue(sum_k A[b,m,k] * B[b,n,k]).
//
// Replaces rocBLAS gemm_ex / gemm_strided_batched_ex behind PyFlame's ROCm
// executor (rocm_blas.cpp:75-153, called from rocm_executor.cpp:278-335) and
// the fused bias/activation epilogues of rocm_kernels.hip:649-732.
//
// Structure (one 128 x BN output tile per CTA, 192 threads):
//   warp 0      TMA producer: K-major 128-byte-swizzled tiles of A and B into a
//               ring of shared-memory stages, completion on mbarriers.
//   warp 1      TMEM allocator and MMA issuer: one elected thread issues
//               tcgen05.mma (kind::tf32 x3 for split-fp32 operands, or
//               kind::f16 with bf16 operands) into a TMEM fp32 accumulator and
//               frees each stage with tcgen05.commit.
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//               lanes 32*(w%4)..+31), alpha/bias/folded-BN/activation/residual,
//               global stores.
// Every mbarrier wait is bounded by the global timer; on expiry the kernel
// records PFC_ERR_TIMEOUT in *err, drains its own copies, frees TMEM and exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "../common.hpp"
#include "kernels.hpp"

namespace pfb {

namespace {

constexpr int kBM = 128;
constexpr int kThreads = 192;
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s per wait

struct GemmParams {
  int M, N, nkb, a_batched, b_batched;
  float* c;
  long long c_sb, c_sm, c_sn;
  float alpha;
  const float* alpha_ptr;
  const float* bias;
  const float* bias_scalar;
  const float* scale;
  const float* shift;
  int act;
  const float* res;
  long long r_sb, r_sm, r_sn;
  int* err;
  int num_m, num_n;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false (and *err set) if the phase did not complete in time.
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity, int* err) {
  if (mbar_try(a, parity)) return true;
  unsigned long long t0 = gtimer();
  while (true) {
    for (int i = 0; i < 128; ++i)
      if (mbar_try(a, parity)) return true;
    if (*(volatile int*)err != 0) return false;
    if (gtimer() - t0 > kWaitNs) {
      atomicCAS(err, 0, PFC_ERR_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t mbar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(mbar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;               // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;     // SBO
  d |= (uint64_t)1 << 46;               // version
  d |= (uint64_t)2 << 61;               // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::tf32 / kind::f16: D fp32, K-major A and B.
__host__ __device__ constexpr uint32_t idesc(int M, int N, uint32_t ab_fmt) {
  return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

template <int PREC>
__device__ __forceinline__ void umma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t id, uint32_t acc) {
  if constexpr (PREC == PFC_PRECISION_BF16) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(da), "l"(db), "r"(id), "r"(acc));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(da), "l"(db), "r"(id), "r"(acc));
  }
}

__device__ __forceinline__ void umma_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float act_apply(float v, int act) {
  switch (act) {
    case 1: return (0.f < v) ? v : 0.f;
    case 2: return 0.5f * v * (1.0f + tanhf(0.7978845608f * (v + 0.044715f * v * v * v)));
    case 3: return 1.0f / (1.0f + expf(-v));
    case 4: return tanhf(v);
    case 5: return v / (1.0f + expf(-v));
    default: return v;
  }
}

template <int PREC, int BN>
struct Cfg {
  static constexpr int ESZ = PREC == PFC_PRECISION_BF16 ? 2 : 4;
  static constexpr int BK = 128 / ESZ;
  static constexpr int UK = PREC == PFC_PRECISION_BF16 ? 16 : 8;
  static constexpr int KSTEPS = BK / UK;
  static constexpr int NOPS = PREC == PFC_PRECISION_BF16 ? 1 : 2;
  static constexpr int A_TILE = kBM * 128;
  static constexpr int B_TILE = BN * 128;
  static constexpr int STAGE = NOPS * (A_TILE + B_TILE);
  static constexpr int STAGES = (200 * 1024) / STAGE > 8 ? 8 : (200 * 1024) / STAGE;
  static constexpr int SMEM = STAGES * STAGE + 1024 /*barriers*/ + 1024 /*align*/;
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr uint32_t IDESC = idesc(kBM, BN, PREC == PFC_PRECISION_BF16 ? 1u : 2u);
};

template <int PREC, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
                const GemmParams p) {
  using C = Cfg<PREC, BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + C::STAGES * C::STAGE);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::STAGES;
  uint64_t* accum = bars + 2 * C::STAGES;
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * C::STAGES + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // an earlier CTA gave up: stop early (block-uniform decision)
  __shared__ int s_stop;
  if (threadIdx.x == 0) s_stop = *(volatile int*)p.err;
  __syncthreads();
  if (s_stop != 0) return;

  // tile coordinates: grouped rasterization (16 M-tiles per group) for L2 reuse
  const int t = blockIdx.x;
  const int group = 16;
  const int per_group = group * p.num_n;
  const int first_m = (t / per_group) * group;
  const int gsz = min(p.num_m - first_m, group);
  const int tm = first_m + (t % per_group) % gsz;
  const int tn = (t % per_group) / gsz;
  const int bz = blockIdx.y;
  const int m0 = tm * kBM, n0 = tn * BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(accum), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  const int nkb = p.nkb;
  bool aborted = false;
  if (warp == 0 && lane == 0) {
    // ---------------- producer ----------------
    const int ca = p.a_batched ? bz : 0, cb = p.b_batched ? bz : 0;
    int issued = 0;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % C::STAGES;
      const uint32_t ph = (uint32_t)(kb / C::STAGES) & 1u;
      if (kb >= C::STAGES && !mbar_wait(smem_u32(&empty[s]), ph ^ 1u, p.err)) { aborted = true; break; }
      uint8_t* st = smem + s * C::STAGE;
      const uint32_t fb = smem_u32(&full[s]);
      mbar_expect_tx(fb, C::STAGE);
      const int kc = kb * C::BK;
      tma_load_3d(smem_u32(st), &ta_hi, fb, kc, m0, ca);
      tma_load_3d(smem_u32(st + C::A_TILE), &tb_hi, fb, kc, n0, cb);
      if constexpr (C::NOPS == 2) {
        tma_load_3d(smem_u32(st + C::A_TILE + C::B_TILE), &ta_lo, fb, kc, m0, ca);
        tma_load_3d(smem_u32(st + 2 * C::A_TILE + C::B_TILE), &tb_lo, fb, kc, n0, cb);
      }
      issued = kb + 1;
    }
    // drain: every issued copy must have landed before the CTA can exit
    for (int kb = issued > C::STAGES ? issued - C::STAGES : 0; kb < issued; ++kb)
      mbar_wait(smem_u32(&full[kb % C::STAGES]), (uint32_t)(kb / C::STAGES) & 1u, p.err);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % C::STAGES;
      const uint32_t ph = (uint32_t)(kb / C::STAGES) & 1u;
      if (!mbar_wait(smem_u32(&full[s]), ph, p.err)) { aborted = true; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t st = smem_u32(smem + s * C::STAGE);
      const uint32_t a_hi = st, b_hi = st + C::A_TILE;
      const uint32_t a_lo = st + C::A_TILE + C::B_TILE, b_lo = st + 2 * C::A_TILE + C::B_TILE;
#pragma unroll
      for (int ks = 0; ks < C::KSTEPS; ++ks) {
        const uint32_t koff = ks * 32;  // 32 bytes of K per instruction
        const uint32_t acc = (kb > 0 || ks > 0) ? 1u : 0u;
        if constexpr (C::NOPS == 2) {
          // small products first, then the leading term
          umma<PREC>(tmem, sdesc(a_lo + koff), sdesc(b_hi + koff), C::IDESC, acc);
          umma<PREC>(tmem, sdesc(a_hi + koff), sdesc(b_lo + koff), C::IDESC, 1u);
          umma<PREC>(tmem, sdesc(a_hi + koff), sdesc(b_hi + koff), C::IDESC, 1u);
        } else {
          umma<PREC>(tmem, sdesc(a_hi + koff), sdesc(b_hi + koff), C::IDESC, acc);
        }
      }
      umma_commit(smem_u32(&empty[s]));
    }
    // signal the epilogue (also after an abort, so in-flight MMAs are tracked)
    umma_commit(smem_u32(accum));
  } else if (warp >= 2) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    bool ok = true;
    if (nkb > 0) ok = mbar_wait(smem_u32(accum), 0u, p.err);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int row = m0 + q * 32 + lane;
    const float alpha = p.alpha_ptr ? *p.alpha_ptr : p.alpha;
    const float bsc = p.bias_scalar ? *p.bias_scalar : 0.f;
    if (ok && *(volatile int*)p.err == 0) {
      float* crow = p.c + (long long)bz * p.c_sb + (long long)row * p.c_sm;
      const float* rrow = p.res ? p.res + (long long)bz * p.r_sb + (long long)row * p.r_sm : nullptr;
#pragma unroll 1
      for (int cc = 0; cc < BN; cc += 16) {
        uint32_t r[16];
        if (nkb > 0) {
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)cc, r);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) r[j] = 0u;
        }
        if (row < p.M) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int n = n0 + cc + j;
            if (n < p.N) {
              float v = __uint_as_float(r[j]);
              if (p.scale) v = v * p.scale[n] + p.shift[n];
              else {
                v = v * alpha;
                if (p.bias) v = v + p.bias[n];
                else if (p.bias_scalar) v = v + bsc;
              }
              v = act_apply(v, p.act);
              if (rrow) v = v + rrow[(long long)n * p.r_sn];
              crow[(long long)n * p.c_sn] = v;
            }
          }
        }
      }
    }
  }
  // teardown: all tcgen05 traffic of this CTA is complete once the epilogue
  // observed `accum` (or gave up); release TMEM.
  (void)aborted;
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS));
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (the
// library does not link libcuda).
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    PFB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    if (!ptr || q != cudaDriverEntryPointSuccess) fail(PFC_ERR_CUDA, "cuTensorMapEncodeTiled not available");
    fn = (EncodeFn)ptr;
  }
  return fn;
}

// 3-D map over a prepared operand [batch][rows][kpad], box (128 bytes of K) x box_rows x 1.
CUtensorMap make_map(const void* base, int prec, int64_t kpad, int64_t rows, int64_t batch, int box_rows) {
  CUtensorMap m;
  std::memset(&m, 0, sizeof m);
  if (!base) return m;
  const int esz = prec == PFC_PRECISION_BF16 ? 2 : 4;
  cuuint64_t dims[3] = {(cuuint64_t)kpad, (cuuint64_t)rows, (cuuint64_t)std::max<int64_t>(batch, 1)};
  cuuint64_t strides[2] = {(cuuint64_t)(kpad * esz), (cuuint64_t)(kpad * rows * esz)};
  cuuint32_t box[3] = {(cuuint32_t)(128 / esz), (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = get_encode()(&m, prec == PFC_PRECISION_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                            3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(PFC_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

template <int PREC, int BN>
void launch_t(const GemmLaunch& L, cudaStream_t stream) {
  using C = Cfg<PREC, BN>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    PFB_CUDA(cudaFuncSetAttribute(gemm_kernel<PREC, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_set[dev & 63] = true;
  }
  const int64_t a_rows = L.M, b_rows = L.N;
  CUtensorMap ta_hi = make_map(L.a_hi, PREC, L.kpad, a_rows, L.a_sb ? L.batch : 1, kBM);
  CUtensorMap tb_hi = make_map(L.b_hi, PREC, L.kpad, b_rows, L.b_sb ? L.batch : 1, BN);
  CUtensorMap ta_lo = PREC == PFC_PRECISION_BF16 ? ta_hi : make_map(L.a_lo, PREC, L.kpad, a_rows, L.a_sb ? L.batch : 1, kBM);
  CUtensorMap tb_lo = PREC == PFC_PRECISION_BF16 ? tb_hi : make_map(L.b_lo, PREC, L.kpad, b_rows, L.b_sb ? L.batch : 1, BN);
  GemmParams p;
  p.M = (int)L.M;
  p.N = (int)L.N;
  p.nkb = (int)(L.kpad / C::BK);
  p.a_batched = L.a_sb != 0;
  p.b_batched = L.b_sb != 0;
  p.c = L.c;
  p.c_sb = L.c_sb;
  p.c_sm = L.c_sm;
  p.c_sn = L.c_sn;
  p.alpha = L.alpha;
  p.alpha_ptr = L.alpha_ptr;
  p.bias = L.bias;
  p.bias_scalar = L.bias_scalar;
  p.scale = L.scale;
  p.shift = L.shift;
  p.act = L.act;
  p.res = L.residual;
  p.r_sb = L.r_sb;
  p.r_sm = L.r_sm;
  p.r_sn = L.r_sn;
  p.err = L.err;
  p.num_m = (int)ceil_div(L.M, kBM);
  p.num_n = (int)ceil_div(L.N, BN);
  if (L.K == 0) p.nkb = 0;
  dim3 grid((unsigned)(p.num_m * p.num_n), (unsigned)L.batch, 1);
  gemm_kernel<PREC, BN><<<grid, kThreads, C::SMEM, stream>>>(ta_hi, ta_lo, tb_hi, tb_lo, p);
  PFB_CUDA(cudaGetLastError());
}

}  // namespace

void launch_gemm(const GemmLaunch& L, cudaStream_t stream) {
  PFB_CHECK_ARG(L.M > 0 && L.N > 0 && L.batch > 0, "gemm: empty problem");
  PFB_CHECK_ARG(L.M < (1ll << 31) && L.N < (1ll << 31), "gemm: dimension too large");
  PFB_CHECK_ARG(L.err != nullptr, "gemm: error flag pointer required");
  const int64_t kal = L.precision == PFC_PRECISION_BF16 ? 64 : 32;
  PFB_CHECK_ARG(L.kpad % kal == 0 && L.kpad >= L.K, "gemm: kpad must be a multiple of the K tile and >= K");
  PFB_CHECK_ARG(((uintptr_t)L.a_hi & 15) == 0 && ((uintptr_t)L.b_hi & 15) == 0, "gemm: operands must be 16-byte aligned");
  if (L.precision == PFC_PRECISION_BF16) {
    if (L.N > 64) launch_t<PFC_PRECISION_BF16, 128>(L, stream);
    else launch_t<PFC_PRECISION_BF16, 64>(L, stream);
  } else {
    PFB_CHECK_ARG(L.a_lo && L.b_lo, "gemm: tf32x3 needs lo operands");
    if (L.N > 64) launch_t<PFC_PRECISION_TF32X3, 128>(L, stream);
    else launch_t<PFC_PRECISION_TF32X3, 64>(L, stream);
  }
}

}  // namespace pfb
