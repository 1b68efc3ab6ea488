// Device helpers shared by the sm_100a tensor-core kernels: mbarrier waits
// bounded by the global timer, TMA tensor loads, shared-memory matrix and
// instruction descriptors, tcgen05.mma issue and commit, TMEM loads.
#pragma once
#include <cuda.h>
#include <cstdint>

#include "../../../include/pyflame_cuda.h"

namespace pfb {
namespace {

constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s per wait

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

// Bounded wait: false (and *err set) if the phase did not complete within
// limit_ns, or if another thread already recorded an error.
__device__ __forceinline__ bool mbar_wait_for(uint32_t a, uint32_t parity, int* err, unsigned long long limit_ns) {
  if (mbar_try(a, parity)) return true;
  unsigned long long t0 = gtimer();
  while (true) {
    for (int i = 0; i < 128; ++i)
      if (mbar_try(a, parity)) return true;
    if (*(volatile int*)err != 0) return false;
    if (gtimer() - t0 > limit_ns) {
      atomicCAS(err, 0, PFC_ERR_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity, int* err) {
  return mbar_wait_for(a, parity, err, kWaitNs);
}

// Bounded wait for a role off the critical path (an epilogue waiting for its
// accumulator): sleeps between tries instead of spinning, which leaves the
// SMSP's issue slots to the warps that share it (the MMA issuer among them).
// Same outcome as mbar_wait: false (and *err set) on timeout or a recorded error.
__device__ __forceinline__ bool mbar_wait_backoff(uint32_t a, uint32_t parity, int* err) {
  if (mbar_try(a, parity)) return true;
  const unsigned long long t0 = gtimer();
  while (true) {
    __nanosleep(256);
    if (mbar_try(a, parity)) return true;
    if (*(volatile int*)err != 0) return false;
    if (gtimer() - t0 > kWaitNs) {
      atomicCAS(err, 0, PFC_ERR_TIMEOUT);
      return false;
    }
  }
}

// Wait for this CTA's own asynchronous work (copies in flight, issued MMAs)
// before its shared memory or TMEM goes away: bounded by time only, even when
// another role already recorded an error.
__device__ __forceinline__ void mbar_wait_own(uint32_t a, uint32_t parity, int* err) {
  if (mbar_try(a, parity)) return;
  unsigned long long t0 = gtimer();
  while (true) {
    for (int i = 0; i < 128; ++i)
      if (mbar_try(a, parity)) return;
    if (gtimer() - t0 > kWaitNs) {
      atomicCAS(err, 0, PFC_ERR_TIMEOUT);
      return;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t mbar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(mbar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t mbar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(mbar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t mbar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(mbar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, uint32_t mbar, int c0, int c1,
                                            int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(mbar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
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

// The 128-byte swizzle is a function of the absolute shared-memory address
// (chunk bits 4-6 XOR row bits 7-9), for TMA writes and tensor-core reads
// alike.  So a matrix may start anywhere on a 16-byte boundary of a swizzled
// buffer: 32 bytes further along K, or a whole number of 128-byte rows
// further down (a tap's run inside a halo), with the plain descriptor and a
// base offset of 0 (verified against the oracle).  Offsets are added to a
// descriptor directly: its low 14 bits hold the address in 16-byte units.
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t bytes) { return d + (bytes >> 4); }

// Descriptor of a K-major operand without swizzle: core matrices of 8 rows x
// 16 bytes, each stored as 128 contiguous bytes (rows 16 bytes apart); lbo =
// bytes from the first to the second 16-byte half of a 32-byte K step, sbo =
// bytes between consecutive 8-row groups.
__device__ __forceinline__ uint64_t sdesc_kint(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // version; layout type 0: no swizzle
  return d;
}

// 1-D bulk copy global -> shared (16-byte aligned addresses, a multiple of
// 16 bytes), completing on the mbarrier's transaction count.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(mbar)
               : "memory");
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

__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void mbar_arrive(uint32_t a) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}

}  // namespace
}  // namespace pfb
