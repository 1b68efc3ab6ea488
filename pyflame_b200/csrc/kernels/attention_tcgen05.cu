// Fused attention for sm_100a: O = softmax(alpha * Q K^T) V over batch x head
// slices, with split-fp32 (3xTF32) operands.
//
// Replaces the three passes PyFlame's MultiheadAttention graph costs behind
// the ROCm executor (rocm_executor.cpp:278-335: a batched GEMM for the
// scores, the softmax kernel of rocm_kernels.hip, a batched GEMM for the
// weighted values), in which the [slices, M, L] scores and probabilities make
// two round trips through HBM.  Here they live in tensor memory only.
//
// One persistent CTA per SM walks tiles of (slice, 128 query rows):
//   warp 0     TMA: Q of the tile once, then key blocks of 64 (K and V)
//              through two-stage rings.
//   warp 1     TMEM (512 columns) and the MMAs, all tf32 x3 as two
//              instructions per K step: the hi x hi and hi x lo products as
//              ONE N = 128 instruction against the concatenated [hi | lo]
//              B operand, then lo x hi (N = 64) into its first half.  (An
//              N = 64 instruction measured ~79 cycles here, about what the
//              N = 128 one costs: 32 wide instructions per key block do the
//              work of 48 narrow ones.)  S = Q K_j^T from shared memory goes
//              into one of two 128-column S/P buffers as [S_hh | S_hl].
//              O_h += P_j,h V_j,h for the two 32-key halves h of the block
//              takes P from the same buffer as the A operand and V as an
//              MN-major B operand (its rows are keys, as stored), into one of
//              two 128-column accumulators [O_hh | O_hl].  The MMAs of a CTA
//              run in issue order, so S_j+2 may be issued into the buffer
//              that P_j*V_j, issued before it, reads.
//   warps 2-9  two warps per TMEM lane quarter; warp half h owns keys
//              32h..32h+31 of every block for its 32 query rows: it reads S
//              (the sum of its two halves), keeps a running max m_h and sum
//              l_h, and writes P = exp2(alpha*log2(e)*s - m_h) as hi/lo tf32
//              over the S it read.  m_h moves only when a block's max exceeds
//              it by more than 2^8 (P stays below 256); then O_h and l_h are
//              rescaled once the previous block's P*V has retired.  At the end
//              of a tile the halves combine, O = (O_0 a_0 + O_1 a_1) /
//              (l_0 a_0 + l_1 a_1) with a_h = 2^(m_h - max(m_0, m_1)).
// Keys past L are masked; query rows past M and head columns past d are
// dropped.  Every wait is bounded by the global timer and reports
// PFC_ERR_TIMEOUT through *err.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "../common.hpp"
#include "kernels.hpp"
#include "split.cuh"
#include "tcgen05.cuh"

namespace pfb {

CUtensorMap make_operand_map(const void* base, int prec, int64_t kpad, int64_t rows, int64_t batch, int box_rows,
                             bool mn32 = false);

namespace {

constexpr int kAQ = 128;          // query rows per tile (one per TMEM lane)
constexpr int kAK = 64;           // keys per block
constexpr int kAD = 64;           // head-dim columns of O and rows of V^T
constexpr int kSoftWarps = 8;
constexpr int kAThreads = (2 + kSoftWarps) * 32;

constexpr int kQChunk = kAQ * 128;  // 128 rows x 32 tf32
constexpr int kKChunk = kAK * 128;  // 64 keys x 32 tf32
constexpr int kVChunk = kAK * 128;  // 64 keys x 32 head-dim columns
constexpr int kQBytes = 2 * 2 * kQChunk;    // [hi/lo][k-chunk]
constexpr int kKStage = 2 * 2 * kKChunk;    // [k-chunk][hi/lo]: hi and lo of a chunk adjacent (one N = 128 operand)
constexpr int kVStage = 2 * 2 * kVChunk;    // [hi/lo][head-dim chunk]
constexpr int kStages = 2;
constexpr int kASmem = kQBytes + kStages * (kKStage + kVStage) + 1024 /*barriers*/ + 1024 /*align*/;
// TMEM columns: S/P buffers at 0 and 128 ([S_hh | S_hl], then P hi over the
// first 64 columns and P lo over the next 64); O accumulators of the two key
// halves at 256 and 384, each [O_hh | O_hl].
constexpr uint32_t kTS = 0, kTO = 256, kATmemCols = 512;
constexpr float kRescaleLog2 = 8.f;  // P < 2^8 between rescales
constexpr uint32_t kIdesc = idesc(kAQ, 64, 2u);  // M 128, N 64, tf32
constexpr uint32_t kIdescMnB = kIdesc | (1u << 16);  // ... with B MN-major
constexpr uint32_t kIdescCat = idesc(kAQ, 128, 2u);  // M 128, N 128 over [hi | lo]
constexpr uint32_t kIdescCatMnB = kIdescCat | (1u << 16);

// Shared-memory descriptor of an MN-major tf32 operand, the one layout
// tcgen05 takes for it: the 128-byte swizzle with 32-byte atoms.  Rows of 32
// N-elements (128 bytes) per K index, 4 K-rows per 512-byte atom (SBO to the
// next 4), the next 32 N-elements `lbo` bytes on.
__device__ __forceinline__ uint64_t sdesc_mn(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)(lbo >> 4) << 16;      // LBO: next 32 N-elements
  d |= (uint64_t)(512 >> 4) << 32;      // SBO: next 4 K-rows
  d |= (uint64_t)1 << 46;               // version
  d |= (uint64_t)1 << 61;               // SWIZZLE_128B_BASE32B
  return d;
}

struct AttnParams {
  int batch, M, L, d, nkc, nblk, ntq;
  float alpha;
  const float* alpha_ptr;
  float* c;  // O of slice s = b*heads + h at c + b*c_sb + h*c_sh + m*c_sm + n*c_sn
  int heads;
  long long c_sb, c_sh, c_sm, c_sn;
  float* o_hi;  // O as tf32 hi/lo at the same element offsets (or null)
  float* o_lo;
  int* err;
};

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// D (TMEM) += A (TMEM, K-major: lane = row, column = k) x B (shared memory,
// K-major for IDESC = kIdesc, MN-major for kIdescMnB)
template <uint32_t IDESC>
__device__ __forceinline__ void umma_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t db, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(db), "n"(IDESC), "r"(acc));
}

// Bounded wait taken by every lane of a warp, with one outcome for all of
// them: the warp-collective TMEM accesses that follow run on all lanes or
// none.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t a, uint32_t parity, int* err) {
  return __all_sync(0xffffffffu, mbar_wait(a, parity, err));
}

// 32 fp32 columns of this warp's TMEM lanes
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
#pragma unroll
  for (int i = 0; i < 2; ++i) tmem_ld16_nowait(taddr + 16 * i, *reinterpret_cast<uint32_t(*)[16]>(&r[16 * i]));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 2^x by the tensor-free special-function unit; results below 2^-126 flush
// to 0 (they are below P's rounding in the sum of a row).
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max of 32 values as a tree (depth 5 instead of a chain of 31); NaN
// entries are ignored as fmaxf ignores them
__device__ __forceinline__ float max32(const float (&v)[32]) {
  float a[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) a[k] = fmaxf(v[k], v[k + 16]);
#pragma unroll
  for (int w = 8; w > 0; w >>= 1)
#pragma unroll
    for (int k = 0; k < w; ++k) a[k] = fmaxf(a[k], a[k + w]);
  return a[0];
}

// 32 fp32 columns at taddr plus the 32 at taddr + step
__device__ __forceinline__ void tmem_ld32_sum(uint32_t taddr, uint32_t step, float (&v)[32]) {
  uint32_t r[32], r2[32];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    tmem_ld16_nowait(taddr + 16 * i, *reinterpret_cast<uint32_t(*)[16]>(&r[16 * i]));
    tmem_ld16_nowait(taddr + step + 16 * i, *reinterpret_cast<uint32_t(*)[16]>(&r2[16 * i]));
  }
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) + __uint_as_float(r2[i]);
}

// Barrier among the softmax warps only.  Every softmax warp passes the same
// barriers in the same order, also after a failed wait: a warp never leaves
// the tile loop except right after softmax_bar_any has told all of them.
__device__ __forceinline__ void softmax_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kSoftWarps * 32) : "memory");
}
// ... and returns whether any softmax thread passed `v` true
__device__ __forceinline__ bool softmax_bar_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kSoftWarps * 32)
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(kAThreads, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tq_hi, const __grid_constant__ CUtensorMap tq_lo,
                const __grid_constant__ CUtensorMap tk_hi, const __grid_constant__ CUtensorMap tk_lo,
                const __grid_constant__ CUtensorMap tv_hi, const __grid_constant__ CUtensorMap tv_lo,
                const AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sq = smem;
  uint8_t* sk = sq + kQBytes;
  uint8_t* sv = sk + kStages * kKStage;
  uint64_t* bars = (uint64_t*)(sv + kStages * kVStage);
  uint64_t* q_full = bars + 0;
  uint64_t* q_free = bars + 1;   // the tile's last S MMAs have read Q
  uint64_t* k_full = bars + 2;   // [2]
  uint64_t* k_free = bars + 4;   // [2]
  uint64_t* v_full = bars + 6;   // [2]
  uint64_t* v_free = bars + 8;   // [2]
  uint64_t* s_full = bars + 10;  // [2] S block in TMEM
  uint64_t* p_full = bars + 14;  // [2] P block written
  uint64_t* p_free = bars + 16;  // [2] P block consumed by its MMAs
  uint64_t* o_full = bars + 18;
  uint64_t* o_free = bars + 19;
  uint64_t* done = bars + 20;
  uint32_t* tmem_slot = (uint32_t*)(bars + 21);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int s_stop;
  if (threadIdx.x == 0) s_stop = *(volatile int*)p.err;
  __syncthreads();
  if (s_stop != 0) return;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    mbar_init(smem_u32(q_free), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&k_full[i]), 1);
      mbar_init(smem_u32(&k_free[i]), 1);
      mbar_init(smem_u32(&v_full[i]), 1);
      mbar_init(smem_u32(&v_free[i]), 1);
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&p_full[i]), kSoftWarps);
      mbar_init(smem_u32(&p_free[i]), 1);
    }
    mbar_init(smem_u32(o_full), 1);
    mbar_init(smem_u32(o_free), kSoftWarps);
    mbar_init(smem_u32(done), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kATmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  const int ntiles = p.batch * p.ntq;
  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    int gk = 0, gv = 0, tc = 0;
    bool ok = true;
    const uint32_t kbytes = (uint32_t)(2 * p.nkc * kKChunk);
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tc) {
      const int b = t / p.ntq, q0 = (t - b * p.ntq) * kAQ;
      if (tc > 0 && !mbar_wait(smem_u32(q_free), (uint32_t)(tc - 1) & 1u, p.err)) { ok = false; break; }
      mbar_expect_tx(smem_u32(q_full), (uint32_t)(2 * p.nkc * kQChunk));
      for (int c = 0; c < p.nkc; ++c) {
        tma_load_3d(smem_u32(sq + c * kQChunk), &tq_hi, smem_u32(q_full), c * 32, q0, b);
        tma_load_3d(smem_u32(sq + (2 + c) * kQChunk), &tq_lo, smem_u32(q_full), c * 32, q0, b);
      }
      {
        for (int j = 0; j < p.nblk; ++j) {
          const int s = gk & 1;
          if (gk >= 2 && !mbar_wait(smem_u32(&k_free[s]), (uint32_t)((gk >> 1) - 1) & 1u, p.err)) { ok = false; break; }
          uint8_t* kst = sk + s * kKStage;
          mbar_expect_tx(smem_u32(&k_full[s]), kbytes);
          for (int c = 0; c < p.nkc; ++c) {
            tma_load_3d(smem_u32(kst + 2 * c * kKChunk), &tk_hi, smem_u32(&k_full[s]), c * 32, j * kAK, b);
            tma_load_3d(smem_u32(kst + (2 * c + 1) * kKChunk), &tk_lo, smem_u32(&k_full[s]), c * 32, j * kAK, b);
          }
          ++gk;
          {
            const int v = gv & 1;
            if (gv >= 2 && !mbar_wait(smem_u32(&v_free[v]), (uint32_t)((gv >> 1) - 1) & 1u, p.err)) { ok = false; break; }
            uint8_t* vst = sv + v * kVStage;
            mbar_expect_tx(smem_u32(&v_full[v]), (uint32_t)kVStage);
            for (int c = 0; c < 2; ++c) {  // head-dim columns 32c..32c+31 of keys j*64..
              tma_load_3d(smem_u32(vst + c * kVChunk), &tv_hi, smem_u32(&v_full[v]), c * 32, j * kAK, b);
              tma_load_3d(smem_u32(vst + (2 + c) * kVChunk), &tv_lo, smem_u32(&v_full[v]), c * 32, j * kAK, b);
            }
            ++gv;
          }
        }
      }
    }
    // drain: every copy issued must land before the CTA exits
    if (tc > 0) mbar_wait_own(smem_u32(q_full), (uint32_t)(tc - 1) & 1u, p.err);
    for (int k = gk > 2 ? gk - 2 : 0; k < gk; ++k) mbar_wait_own(smem_u32(&k_full[k & 1]), (uint32_t)(k >> 1) & 1u, p.err);
    for (int k = gv > 2 ? gv - 2 : 0; k < gv; ++k) mbar_wait_own(smem_u32(&v_full[k & 1]), (uint32_t)(k >> 1) & 1u, p.err);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    int gk = 0, gv = 0, gs = 0, gp = 0, tc = 0;
    bool ok = true;
    const uint32_t q_base = smem_u32(sq);
    // S[gs & 1] = Q K^T of the next K block.  Its buffer last held P of
    // block gs-2, whose P*V MMAs were issued before these.
    auto issue_s = [&]() -> bool {
      const int sb = gs & 1, ks = gk & 1;
      if (!mbar_wait(smem_u32(&k_full[ks]), (uint32_t)(gk >> 1) & 1u, p.err)) return false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t d = tmem + kTS + (uint32_t)(sb * 128);
      const uint32_t k_base = smem_u32(sk + ks * kKStage);
      for (int c = 0; c < p.nkc; ++c) {
        const uint64_t qh = sdesc(q_base + c * kQChunk), ql = sdesc(q_base + (2 + c) * kQChunk);
        const uint64_t khl = sdesc(k_base + 2 * c * kKChunk);  // [K_hi | K_lo]; its first 64 rows are K_hi
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t off = kk * 32;
          const uint32_t acc = (c > 0 || kk > 0) ? 1u : 0u;
          umma<PFC_PRECISION_TF32X3>(d, desc_add(qh, off), desc_add(khl, off), kIdescCat, acc);
          umma<PFC_PRECISION_TF32X3>(d, desc_add(ql, off), desc_add(khl, off), kIdesc, 1u);
        }
      }
      umma_commit(smem_u32(&k_free[ks]));
      umma_commit(smem_u32(&s_full[sb]));
      ++gk;
      ++gs;
      return true;
    };
    // O += P V of key block j
    auto issue_pv = [&](int j) -> bool {
      const int pb = gp & 1, vs = gv & 1;
      if (!mbar_wait(smem_u32(&p_full[pb]), (uint32_t)(gp >> 1) & 1u, p.err)) return false;
      if (!mbar_wait(smem_u32(&v_full[vs]), (uint32_t)(gv >> 1) & 1u, p.err)) return false;
      if (j == 0 && tc > 0 && !mbar_wait(smem_u32(o_free), (uint32_t)(tc - 1) & 1u, p.err)) return false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t ph = tmem + kTS + (uint32_t)(pb * 128), pl = ph + 64;
      const uint32_t v_base = smem_u32(sv + vs * kVStage);
      // V block [64 keys][64 head dims] as 32-column chunks [hi 0][hi 1]
      // [lo 0][lo 1], LBO apart: one descriptor spans N = 128 ([V_hi | V_lo])
      // or, at N = 64, V_hi.  K-step kk takes keys 8kk..8kk+7 (one 1024-byte
      // row group further down); keys 32h.. go to accumulator O_h
      const uint64_t vhl = sdesc_mn(v_base, kVChunk);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t d = tmem + kTO + (uint32_t)(h * 128);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t col = (uint32_t)(h * 32 + kk * 8), off = (uint32_t)(h * 4 + kk) * 1024u;
          const uint32_t acc = (j > 0 || kk > 0) ? 1u : 0u;
          umma_tmem_a<kIdescCatMnB>(d, ph + col, desc_add(vhl, off), acc);
          umma_tmem_a<kIdescMnB>(d, pl + col, desc_add(vhl, off), 1u);
        }
      }
      umma_commit(smem_u32(&v_free[vs]));
      umma_commit(smem_u32(&p_free[pb]));
      ++gv;
      ++gp;
      return true;
    };
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tc) {
      if (!mbar_wait(smem_u32(q_full), (uint32_t)tc & 1u, p.err)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      // S of the next block goes in before P V of this one, so the softmax
      // warps work on one block while the tensor core does the other
      ok = issue_s();
      for (int j = 0; j < p.nblk && ok; ++j) {
        if (j + 1 < p.nblk) ok = issue_s();
        if (ok && j + 1 == p.nblk) umma_commit(smem_u32(q_free));  // the last S of the tile is issued
        if (ok) ok = issue_pv(j);
      }
      if (ok) umma_commit(smem_u32(o_full));
    }
    umma_commit(smem_u32(done));
  } else if (warp >= 2) {
    // ---------------- softmax and output ----------------
    __shared__ float2 row_stat[2][kAQ];  // (max, sum) of each half of a row
    const int q = warp & 3, hf = (warp - 2) >> 2;
    const int row_in_tile = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const float scale = (p.alpha_ptr ? *p.alpha_ptr : p.alpha) * 1.4426950408889634f;  // alpha * log2(e)
    int gs = 0, gp = 0, tc = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tc) {
      const int b = t / p.ntq, q0 = (t - b * p.ntq) * kAQ;
      float m = -INFINITY, l = 0.f;
      float v[32];
      // this warp's 32 keys of S: the sum of the hi x hi and hi x lo halves
      // (the lo x hi product is in the first)
      auto read_s = [&]() -> bool {
        const int sb = gs & 1;
        if (!mbar_wait_warp(smem_u32(&s_full[sb]), (uint32_t)(gs >> 1) & 1u, p.err)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        tmem_ld32_sum(lane_base + kTS + (uint32_t)(sb * 128 + hf * 32), 64u, v);
        ++gs;
        return true;
      };
      // one pass: this half's keys, running max m (log2 units, moved lazily)
      // and sum l of P = exp2(scale * s - m)
      for (int j = 0; j < p.nblk && ok; ++j) {
        if (!(ok = read_s())) break;
        const int nk = min(32, p.L - j * kAK - hf * 32);
        // scores in log2 units; keys past L (last block only) drop out of
        // the max and get P = 2^-inf = 0
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] *= scale;
        if (nk < 32) {
#pragma unroll
          for (int k = 0; k < 32; ++k)
            if (k >= nk) v[k] = -INFINITY;
        }
        const float bm = max32(v);
        const bool first = m == -INFINITY;
        const bool move = bm > (first ? -INFINITY : m + kRescaleLog2);
        const float mn = move ? bm : m;
        if (__any_sync(0xffffffffu, move && !first && j > 0)) {
          // O_h holds blocks up to j-1: wait for their P*V, then rescale
          const int prev = gp - 1;
          if (!(ok = mbar_wait_warp(smem_u32(&p_free[prev & 1]), (uint32_t)(prev >> 1) & 1u, p.err))) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const float a = (move && !first) ? exp2f(m - mn) : 1.f;
          const uint32_t oaddr = lane_base + kTO + (uint32_t)(hf * 128);
          float o[32];
#pragma unroll
          for (int c = 0; c < 128; c += 32) {
            tmem_ld32(oaddr + c, o);
            uint32_t w[32];
#pragma unroll
            for (int k = 0; k < 32; ++k) w[k] = __float_as_uint(o[k] * a);
            tmem_st16(oaddr + c, *reinterpret_cast<const uint32_t(*)[16]>(&w[0]));
            tmem_st16(oaddr + c + 16, *reinterpret_cast<const uint32_t(*)[16]>(&w[16]));
          }
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        if (move && !first) l *= exp2f(m - mn);
        m = mn;
        // P over the S just read (hi) and beside it (lo); the buffer's
        // previous P was consumed before this S was computed into it
        const int pb = gp & 1;
        const uint32_t pbase = lane_base + kTS + (uint32_t)(pb * 128 + hf * 32);
        const float msub = m == -INFINITY ? 0.f : m;  // a half with no keys yet: every P is 0
        float sum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float pv = ex2_ftz(v[16 * i + k] - msub);
            sum[k & 3] += pv;
            // P is finite here (0 <= P < 2^8 between rescales); a NaN or
            // infinite score makes lo NaN and with it the row's output
            hi[k] = __float_as_uint(pv) & 0xFFFFE000u;
            lo[k] = __float_as_uint(pv - __uint_as_float(hi[k]));
          }
          tmem_st16(pbase + 16 * i, hi);
          tmem_st16(pbase + 64 + 16 * i, lo);
        }
        l += (sum[0] + sum[1]) + (sum[2] + sum[3]);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&p_full[pb]));
        ++gp;
      }
      // the two halves of the row: weights a_h = 2^(m_h - m) (0 for a half without keys)
      row_stat[hf][row_in_tile] = make_float2(m, l);
      if (softmax_bar_any(!ok)) break;  // all softmax warps leave together
      float a_self, a_other, inv;
      {
        const float2 o = row_stat[hf ^ 1][row_in_tile];
        const float mx = fmaxf(m, o.x);
        a_self = m == -INFINITY ? 0.f : exp2f(m - mx);
        a_other = o.x == -INFINITY ? 0.f : exp2f(o.x - mx);
        inv = 1.f / (l * a_self + o.y * a_other);
      }
      softmax_bar();  // row_stat is free for the next tile
      const float a0 = (hf == 0 ? a_self : a_other) * inv, a1 = (hf == 0 ? a_other : a_self) * inv;
      // From here a failed wait skips the rest of this tile; the warp still
      // meets the others at the next tile's barrier, which ends the loop.
      if (!ok) continue;
      // this warp's half of the output row
      if (!(ok = mbar_wait_warp(smem_u32(o_full), (uint32_t)tc & 1u, p.err))) continue;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      {
        float o1[32];
        tmem_ld32_sum(lane_base + kTO + (uint32_t)(hf * 32), 64u, v);           // O_0, this warp's 32 columns
        tmem_ld32_sum(lane_base + kTO + 128u + (uint32_t)(hf * 32), 64u, o1);  // O_1, the same columns
#pragma unroll
        for (int n = 0; n < 32; ++n) v[n] = v[n] * a0 + o1[n] * a1;
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(o_free));
      const int row = q0 + row_in_tile;
      if (row < p.M) {
        const int bb = b / p.heads, hh = b - bb * p.heads;
        const long long off = (long long)bb * p.c_sb + (long long)hh * p.c_sh + (long long)row * p.c_sm +
                              (long long)(hf * 32) * p.c_sn;
        const bool vec = p.c_sn == 1 && p.d == 64 && (off & 3) == 0;
        if (p.c) {
          float* out = p.c + off;
          if (vec) {
#pragma unroll
            for (int n = 0; n < 32; n += 4)
              *reinterpret_cast<float4*>(out + n) = make_float4(v[n], v[n + 1], v[n + 2], v[n + 3]);
          } else {
#pragma unroll
            for (int n = 0; n < 32; ++n)
              if (hf * 32 + n < p.d) out[(long long)n * p.c_sn] = v[n];
          }
        }
        if (p.o_hi) {
#pragma unroll
          for (int n = 0; n < 32; n += 4) {
            float4 h, lw;
            split_tf32(v[n], h.x, lw.x);
            split_tf32(v[n + 1], h.y, lw.y);
            split_tf32(v[n + 2], h.z, lw.z);
            split_tf32(v[n + 3], h.w, lw.w);
            if (vec) {
              *reinterpret_cast<float4*>(p.o_hi + off + n) = h;
              *reinterpret_cast<float4*>(p.o_lo + off + n) = lw;
            } else {
              const float hs[4] = {h.x, h.y, h.z, h.w}, ls[4] = {lw.x, lw.y, lw.z, lw.w};
              for (int k = 0; k < 4; ++k)
                if (hf * 32 + n + k < p.d) {
                  p.o_hi[off + (long long)(n + k) * p.c_sn] = hs[k];
                  p.o_lo[off + (long long)(n + k) * p.c_sn] = ls[k];
                }
            }
          }
        }
      }
    }
  }
  // teardown: every MMA retired before TMEM is released
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) mbar_wait_own(smem_u32(done), 0u, p.err);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kATmemCols));
  }
}

// ---------------------------------------------------------------------------
// The bf16 mode: the same roles with bf16 operands, one kind::f16 MMA per K
// step (16 elements) and P in TMEM as packed bf16 pairs.
//   warp 0     TMA: Q of the tile ([128 rows][64 bf16], one 128-byte row per
//              query), key blocks of 64 through three-stage K and V rings.
//   warp 1     S = Q K_j^T (4 instructions, M 128, N 64) into one of two
//              64-column S/P buffers; O_h += P_h V_h for the two 32-key halves
//              (2 instructions each, A = P from TMEM, V an MN-major B operand:
//              its 128-byte rows are keys, as stored) into two 64-column
//              accumulators.
//   warps 2-9  as in the tf32 kernel: warp half h reads its 32 keys of S,
//              keeps its running max m_h (moved lazily, 2^8) and sum l_h, and
//              writes P = exp2(alpha*log2(e)*s - m_h) rounded to bf16 as 16
//              packed columns over the first half of the S columns it read;
//              l_h sums the rounded values.  The halves combine per tile.
// O goes out as fp32 and / or as the next GEMM's bf16 operand.
constexpr int kBRow = 128;                  // bytes per row: 64 bf16
constexpr int kBQBytes = kAQ * kBRow;       // Q tile
constexpr int kBKBytes = kAK * kBRow;       // K block
constexpr int kBVBytes = kAK * kBRow;       // V block [64 keys][64 head dims]
constexpr int kBStages = 3;
constexpr int kBSmem = kBQBytes + kBStages * (kBKBytes + kBVBytes) + 1024 + 1024;
constexpr uint32_t kBTS = 0, kBTO = 128, kBTmemCols = 256;
constexpr uint32_t kBIdesc = idesc(kAQ, 64, 1u);        // M 128, N 64, bf16 -> fp32
constexpr uint32_t kBIdescMnB = kBIdesc | (1u << 16);   // ... with B MN-major

// Shared-memory descriptor of an MN-major bf16 operand in the 128-byte
// swizzle: rows of 64 N-elements (128 bytes) per K index, 8 K-rows per
// 1024-byte atom (SBO to the next 8); one atom column covers N = 64.
__device__ __forceinline__ uint64_t sdesc_mn16(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;                // LBO: a single atom column
  d |= (uint64_t)(1024 >> 4) << 32;      // SBO: next 8 K-rows
  d |= (uint64_t)1 << 46;                // version
  d |= (uint64_t)2 << 61;                // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void umma_tmem_a16(uint32_t d_tmem, uint32_t a_tmem, uint64_t db, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(db), "n"(kBIdescMnB), "r"(acc));
}

__global__ void __launch_bounds__(kAThreads, 1)
    attn_bf16_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, const AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sq = smem;
  uint8_t* sk = sq + kBQBytes;
  uint8_t* sv = sk + kBStages * kBKBytes;
  uint64_t* bars = (uint64_t*)(sv + kBStages * kBVBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* q_free = bars + 1;
  uint64_t* k_full = bars + 2;   // [3]
  uint64_t* k_free = bars + 5;   // [3]
  uint64_t* v_full = bars + 8;   // [3]
  uint64_t* v_free = bars + 11;  // [3]
  uint64_t* s_full = bars + 14;  // [2]
  uint64_t* p_full = bars + 16;  // [2]
  uint64_t* p_free = bars + 18;  // [2]
  uint64_t* o_full = bars + 20;
  uint64_t* o_free = bars + 21;
  uint64_t* done = bars + 22;
  uint32_t* tmem_slot = (uint32_t*)(bars + 23);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int s_stop;
  if (threadIdx.x == 0) s_stop = *(volatile int*)p.err;
  __syncthreads();
  if (s_stop != 0) return;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    mbar_init(smem_u32(q_free), 1);
    for (int i = 0; i < kBStages; ++i) {
      mbar_init(smem_u32(&k_full[i]), 1);
      mbar_init(smem_u32(&k_free[i]), 1);
      mbar_init(smem_u32(&v_full[i]), 1);
      mbar_init(smem_u32(&v_free[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&p_full[i]), kSoftWarps);
      mbar_init(smem_u32(&p_free[i]), 1);
    }
    mbar_init(smem_u32(o_full), 1);
    mbar_init(smem_u32(o_free), kSoftWarps);
    mbar_init(smem_u32(done), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kBTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  const int ntiles = p.batch * p.ntq;
  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    int gk = 0, tc = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tc) {
      const int b = t / p.ntq, q0 = (t - b * p.ntq) * kAQ;
      if (tc > 0 && !mbar_wait(smem_u32(q_free), (uint32_t)(tc - 1) & 1u, p.err)) { ok = false; break; }
      mbar_expect_tx(smem_u32(q_full), (uint32_t)kBQBytes);
      tma_load_3d(smem_u32(sq), &tq, smem_u32(q_full), 0, q0, b);
      for (int j = 0; j < p.nblk; ++j, ++gk) {
        const int s = gk % kBStages;
        const uint32_t use = (uint32_t)(gk / kBStages);
        if (gk >= kBStages && !mbar_wait(smem_u32(&k_free[s]), (use - 1) & 1u, p.err)) { ok = false; break; }
        mbar_expect_tx(smem_u32(&k_full[s]), (uint32_t)kBKBytes);
        tma_load_3d(smem_u32(sk + s * kBKBytes), &tk, smem_u32(&k_full[s]), 0, j * kAK, b);
        if (gk >= kBStages && !mbar_wait(smem_u32(&v_free[s]), (use - 1) & 1u, p.err)) { ok = false; break; }
        mbar_expect_tx(smem_u32(&v_full[s]), (uint32_t)kBVBytes);
        tma_load_3d(smem_u32(sv + s * kBVBytes), &tv, smem_u32(&v_full[s]), 0, j * kAK, b);
      }
    }
    // drain: every copy issued must land before the CTA exits
    if (tc > 0) mbar_wait_own(smem_u32(q_full), (uint32_t)(tc - 1) & 1u, p.err);
    for (int k = gk > kBStages ? gk - kBStages : 0; k < gk; ++k) {
      mbar_wait_own(smem_u32(&k_full[k % kBStages]), (uint32_t)(k / kBStages) & 1u, p.err);
      mbar_wait_own(smem_u32(&v_full[k % kBStages]), (uint32_t)(k / kBStages) & 1u, p.err);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    int gk = 0, gv = 0, gs = 0, gp = 0, tc = 0;
    bool ok = true;
    const uint64_t qd = sdesc(smem_u32(sq));
    // S[gs & 1] = Q K^T of the next key block; its buffer last held P of
    // block gs-2, whose P*V MMAs were issued before these
    auto issue_s = [&]() -> bool {
      const int sb = gs & 1, ks = gk % kBStages;
      if (!mbar_wait(smem_u32(&k_full[ks]), (uint32_t)(gk / kBStages) & 1u, p.err)) return false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t d = tmem + kBTS + (uint32_t)(sb * 64);
      const uint64_t kd = sdesc(smem_u32(sk + ks * kBKBytes));
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma<PFC_PRECISION_BF16>(d, desc_add(qd, kk * 32), desc_add(kd, kk * 32), kBIdesc, kk > 0 ? 1u : 0u);
      umma_commit(smem_u32(&k_free[ks]));
      umma_commit(smem_u32(&s_full[sb]));
      ++gk;
      ++gs;
      return true;
    };
    // O_h += P_h V_h of key block j
    auto issue_pv = [&](int j) -> bool {
      const int pb = gp & 1, vs = gv % kBStages;
      if (!mbar_wait(smem_u32(&p_full[pb]), (uint32_t)(gp >> 1) & 1u, p.err)) return false;
      if (!mbar_wait(smem_u32(&v_full[vs]), (uint32_t)(gv / kBStages) & 1u, p.err)) return false;
      if (j == 0 && tc > 0 && !mbar_wait(smem_u32(o_free), (uint32_t)(tc - 1) & 1u, p.err)) return false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t pbuf = tmem + kBTS + (uint32_t)(pb * 64);
      const uint64_t vd = sdesc_mn16(smem_u32(sv + vs * kBVBytes));
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t d = tmem + kBTO + (uint32_t)(h * 64);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          // keys 32h + 16kk ..: 8 packed P columns, 16 rows of V (2 KB further down)
          const uint32_t col = (uint32_t)(h * 32 + kk * 8), off = (uint32_t)(h * 2 + kk) * 2048u;
          umma_tmem_a16(d, pbuf + col, desc_add(vd, off), (j > 0 || kk > 0) ? 1u : 0u);
        }
      }
      umma_commit(smem_u32(&v_free[vs]));
      umma_commit(smem_u32(&p_free[pb]));
      ++gv;
      ++gp;
      return true;
    };
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tc) {
      if (!mbar_wait(smem_u32(q_full), (uint32_t)tc & 1u, p.err)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      ok = issue_s();
      for (int j = 0; j < p.nblk && ok; ++j) {
        if (j + 1 < p.nblk) ok = issue_s();
        if (ok && j + 1 == p.nblk) umma_commit(smem_u32(q_free));  // the last S of the tile is issued
        if (ok) ok = issue_pv(j);
      }
      if (ok) umma_commit(smem_u32(o_full));
    }
    umma_commit(smem_u32(done));
  } else if (warp >= 2) {
    // ---------------- softmax and output ----------------
    __shared__ float2 row_stat[2][kAQ];  // (max, sum) of each half of a row
    const int q = warp & 3, hf = (warp - 2) >> 2;
    const int row_in_tile = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const float scale = (p.alpha_ptr ? *p.alpha_ptr : p.alpha) * 1.4426950408889634f;  // alpha * log2(e)
    int gs = 0, gp = 0, tc = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tc) {
      const int b = t / p.ntq, q0 = (t - b * p.ntq) * kAQ;
      float m = -INFINITY, l = 0.f;
      float v[32];
      for (int j = 0; j < p.nblk && ok; ++j) {
        const int sb = gs & 1;
        if (!(ok = mbar_wait_warp(smem_u32(&s_full[sb]), (uint32_t)(gs >> 1) & 1u, p.err))) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t sbase = lane_base + kBTS + (uint32_t)(sb * 64 + hf * 32);
        tmem_ld32(sbase, v);
        ++gs;
        const int nk = min(32, p.L - j * kAK - hf * 32);
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] *= scale;
        if (nk < 32) {
#pragma unroll
          for (int k = 0; k < 32; ++k)
            if (k >= nk) v[k] = -INFINITY;
        }
        const float bm = max32(v);
        const bool first = m == -INFINITY;
        const bool move = bm > (first ? -INFINITY : m + kRescaleLog2);
        const float mn = move ? bm : m;
        if (__any_sync(0xffffffffu, move && !first && j > 0)) {
          // O_h holds blocks up to j-1: wait for their P*V, then rescale
          const int prev = gp - 1;
          if (!(ok = mbar_wait_warp(smem_u32(&p_free[prev & 1]), (uint32_t)(prev >> 1) & 1u, p.err))) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const float a = (move && !first) ? exp2f(m - mn) : 1.f;
          const uint32_t oaddr = lane_base + kBTO + (uint32_t)(hf * 64);
          float o[32];
#pragma unroll
          for (int c = 0; c < 64; c += 32) {
            tmem_ld32(oaddr + c, o);
            uint32_t w[32];
#pragma unroll
            for (int k = 0; k < 32; ++k) w[k] = __float_as_uint(o[k] * a);
            tmem_st16(oaddr + c, *reinterpret_cast<const uint32_t(*)[16]>(&w[0]));
            tmem_st16(oaddr + c + 16, *reinterpret_cast<const uint32_t(*)[16]>(&w[16]));
          }
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        if (move && !first) l *= exp2f(m - mn);
        m = mn;
        const int pb = gp & 1;
        const float msub = m == -INFINITY ? 0.f : m;  // a half with no keys yet: every P is 0
        uint32_t pk[16];
        float sum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(ex2_ftz(v[2 * k] - msub), ex2_ftz(v[2 * k + 1] - msub));
          pk[k] = *reinterpret_cast<const uint32_t*>(&h2);
          sum[k & 3] += __low2float(h2) + __high2float(h2);
        }
        // P over the first 16 of the 32 S columns this warp read
        tmem_st16(lane_base + kBTS + (uint32_t)(pb * 64 + hf * 32), pk);
        l += (sum[0] + sum[1]) + (sum[2] + sum[3]);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&p_full[pb]));
        ++gp;
      }
      row_stat[hf][row_in_tile] = make_float2(m, l);
      if (softmax_bar_any(!ok)) break;  // all softmax warps leave together
      float a_self, a_other, inv;
      {
        const float2 o = row_stat[hf ^ 1][row_in_tile];
        const float mx = fmaxf(m, o.x);
        a_self = m == -INFINITY ? 0.f : exp2f(m - mx);
        a_other = o.x == -INFINITY ? 0.f : exp2f(o.x - mx);
        inv = 1.f / (l * a_self + o.y * a_other);
      }
      softmax_bar();  // row_stat is free for the next tile
      const float a0 = (hf == 0 ? a_self : a_other) * inv, a1 = (hf == 0 ? a_other : a_self) * inv;
      if (!ok) continue;
      if (!(ok = mbar_wait_warp(smem_u32(o_full), (uint32_t)tc & 1u, p.err))) continue;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      {
        float o1[32];
        tmem_ld32(lane_base + kBTO + (uint32_t)(hf * 32), v);        // O_0, this warp's 32 columns
        tmem_ld32(lane_base + kBTO + 64u + (uint32_t)(hf * 32), o1);  // O_1, the same columns
#pragma unroll
        for (int n = 0; n < 32; ++n) v[n] = v[n] * a0 + o1[n] * a1;
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(o_free));
      const int row = q0 + row_in_tile;
      if (row < p.M) {
        const int bb = b / p.heads, hh = b - bb * p.heads;
        const long long off = (long long)bb * p.c_sb + (long long)hh * p.c_sh + (long long)row * p.c_sm +
                              (long long)(hf * 32) * p.c_sn;
        const bool vec = p.c_sn == 1 && p.d == 64 && (off & 3) == 0;
        if (p.c) {
          float* out = p.c + off;
          if (vec) {
#pragma unroll
            for (int n = 0; n < 32; n += 4)
              *reinterpret_cast<float4*>(out + n) = make_float4(v[n], v[n + 1], v[n + 2], v[n + 3]);
          } else {
#pragma unroll
            for (int n = 0; n < 32; ++n)
              if (hf * 32 + n < p.d) out[(long long)n * p.c_sn] = v[n];
          }
        }
        if (p.o_hi) {
          __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(p.o_hi) + off;
          if (vec) {
#pragma unroll
            for (int n = 0; n < 32; n += 4) {
              const __nv_bfloat162 a = __floats2bfloat162_rn(v[n], v[n + 1]), c2 = __floats2bfloat162_rn(v[n + 2], v[n + 3]);
              uint2 pk2;
              pk2.x = *reinterpret_cast<const uint32_t*>(&a);
              pk2.y = *reinterpret_cast<const uint32_t*>(&c2);
              *reinterpret_cast<uint2*>(ob + n) = pk2;
            }
          } else {
            for (int n = 0; n < 32; ++n)
              if (hf * 32 + n < p.d) ob[(long long)n * p.c_sn] = __float2bfloat16_rn(v[n]);
          }
        }
      }
    }
  }
  // teardown: every MMA retired before TMEM is released
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) mbar_wait_own(smem_u32(done), 0u, p.err);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kBTmemCols));
  }
}

}  // namespace

void launch_attention(const AttnLaunch& L, cudaStream_t stream) {
  PFB_CHECK_ARG(L.batch > 0 && L.M > 0 && L.L > 0 && L.d > 0, "attention: empty problem");
  const bool bf16 = L.precision == PFC_PRECISION_BF16;
  PFB_CHECK_ARG(L.d <= kAD && (L.kq == 64 || (!bf16 && L.kq == 32)), "attention: head dimensions must be <= 64");
  PFB_CHECK_ARG(L.kv == 64 || (!bf16 && L.kv == 32), "attention: V operand must have 32 or 64 padded head-dim columns");
  PFB_CHECK_ARG(L.batch < (1 << 20) && L.M < (1 << 24) && L.L < (1 << 24), "attention: too large");
  PFB_CHECK_ARG(L.err && (L.c || L.o_hi) && (!L.o_hi || bf16 || L.o_lo) && L.heads > 0 && L.batch % L.heads == 0,
                "attention: null pointer or bad head count");
  PFB_CHECK_ARG(!L.o_hi || (((uintptr_t)L.o_hi | (uintptr_t)L.o_lo) & 15) == 0, "attention: operand output must be 16-byte aligned");
  for (const void* q : {L.q_hi, (const void*)L.q_lo, L.k_hi, (const void*)L.k_lo, L.v_hi, (const void*)L.v_lo})
    PFB_CHECK_ARG((bf16 && (q == L.q_lo || q == L.k_lo || q == L.v_lo)) || (q && ((uintptr_t)q & 15) == 0),
                  "attention: operands must be 16-byte aligned");
  // per-device set-up once, safe when several host threads launch at once
  static std::once_flag attr_once[64];
  const int dev = current_device();
  std::call_once(attr_once[dev], [] {
    PFB_CUDA(cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kASmem));
    PFB_CUDA(cudaFuncSetAttribute(attn_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBSmem));
  });
  const int n_sms = device_sm_count(dev);
  const int prec = PFC_PRECISION_TF32X3;
  AttnParams p;
  p.batch = (int)L.batch;
  p.M = (int)L.M;
  p.L = (int)L.L;
  p.d = (int)L.d;
  p.nkc = (int)(L.kq / 32);
  p.nblk = (int)ceil_div(L.L, kAK);
  p.ntq = (int)ceil_div(L.M, kAQ);
  p.alpha = L.alpha;
  p.alpha_ptr = L.alpha_ptr;
  p.c = L.c;
  p.heads = (int)L.heads;
  p.c_sb = L.c_sb;
  p.c_sh = L.c_sh;
  p.c_sm = L.c_sm;
  p.c_sn = L.c_sn;
  p.o_hi = L.o_hi;
  p.o_lo = L.o_lo;
  p.err = L.err;
  const int64_t ntiles = (int64_t)p.batch * p.ntq;
  PFB_CHECK_ARG(ntiles < (1ll << 31), "attention: too many tiles");
  const unsigned grid = (unsigned)std::min<int64_t>(ntiles, n_sms);
  if (bf16) {
    const CUtensorMap q = make_operand_map(L.q_hi, PFC_PRECISION_BF16, 64, L.M, L.batch, kAQ);
    const CUtensorMap k = make_operand_map(L.k_hi, PFC_PRECISION_BF16, 64, L.L, L.batch, kAK);
    // V rows are keys of 64 head dims: read as stored, an MN-major operand
    const CUtensorMap v = make_operand_map(L.v_hi, PFC_PRECISION_BF16, 64, L.L, L.batch, kAK);
    attn_bf16_kernel<<<grid, kAThreads, kBSmem, stream>>>(q, k, v, p);
    PFB_CUDA(cudaGetLastError());
    return;
  }
  const CUtensorMap qh = make_operand_map(L.q_hi, prec, L.kq, L.M, L.batch, kAQ);
  const CUtensorMap ql = make_operand_map(L.q_lo, prec, L.kq, L.M, L.batch, kAQ);
  const CUtensorMap kh = make_operand_map(L.k_hi, prec, L.kq, L.L, L.batch, kAK);
  const CUtensorMap kl = make_operand_map(L.k_lo, prec, L.kq, L.L, L.batch, kAK);
  const CUtensorMap vh = make_operand_map(L.v_hi, prec, L.kv, L.L, L.batch, kAK, true);
  const CUtensorMap vl = make_operand_map(L.v_lo, prec, L.kv, L.L, L.batch, kAK, true);
  attn_kernel<<<grid, kAThreads, kASmem, stream>>>(qh, ql, kh, kl, vh, vl, p);
  PFB_CUDA(cudaGetLastError());
}

}  // namespace pfb
