// Tensor-core GEMM for sm_100a: C[b,m,n] = epilogue(sum_k A[b,m,k] * B[b,n,k]).
//
// Replaces rocBLAS gemm_ex / gemm_strided_batched_ex behind PyFlame's ROCm
// executor (rocm_blas.cpp:75-153, called from rocm_executor.cpp:278-335) and
// the fused bias/activation epilogues of rocm_kernels.hip:649-732.
//
// Structure: a persistent kernel, one CTA of 320 threads per SM, each CTA
// walking 128 x BN output tiles (tile blockIdx.x, +gridDim.x, ...):
//   warp 0      TMA producer: K-major 128-byte-swizzled tiles of A and B into a
//               ring of shared-memory stages, completion on mbarriers; the
//               ring runs on across tile boundaries.  (Implicit-GEMM Conv2d:
//               warps 0..3 gather A rows instead, and the roles below shift
//               up by three warps.)
//   warp 1      TMEM allocator and MMA issuer: one elected thread issues
//               tcgen05.mma (kind::tf32 x3 for split-fp32 operands, or
//               kind::f16 with bf16 operands) into one of two TMEM fp32
//               accumulators and frees each stage with tcgen05.commit.
//   warps 2..9  epilogue, two warps per TMEM lane quarter (warp w reads
//               lanes 32*(w%4)..+31), each taking half of the tile's
//               columns: tcgen05.ld of each finished accumulator into fp32
//               registers, returned at once to the MMA warp; once a tile's K
//               is complete, 32x16 blocks go through shared memory so that a
//               warp stores 8 rows x 16 consecutive columns per float4 pass,
//               applying alpha/bias/folded-BN/activation/residual.  With two
//               accumulators the epilogue of tile i overlaps the MMAs of i+1.
// K is accumulated in chunks of 512 elements, each into a fresh accumulator,
// and the chunks are summed in fp32 registers: a long accumulation inside the
// tensor core drifts (at K = 16384 by about 1e-4 of the row scale, always
// toward zero), a chunk of 512 stays well inside fp32-reference accuracy.
// Every mbarrier wait is bounded by the global timer; on expiry the kernel
// records PFC_ERR_TIMEOUT in *err, drains its own copies, waits for its own
// MMAs to retire, frees TMEM and exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include <cuda_bf16.h>

#include "../common.hpp"
#include "kernels.hpp"
#include "split.cuh"
#include "act.cuh"
#include "tcgen05.cuh"

namespace pfb {

namespace {

constexpr int kBM = 128;
// Warps: producers (1 TMA warp, or 4 gathering warps for CONV), 1 MMA warp,
// 8 epilogue warps (two per TMEM lane quarter, each taking half the columns).
constexpr int kEpiWarps = 8;
template <bool CONV>
constexpr int kProdWarps = CONV ? 4 : 1;
template <bool CONV>
constexpr int kThreads = (kProdWarps<CONV> + 1 + kEpiWarps) * 32;

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
  int num_m, num_n, batch;
  int kchunk, nchunks;  // k-blocks per accumulation chunk; chunks per tile
  void* o_hi;           // operand outputs for a following GEMM (or null)
  float* o_lo;
  long long o_sm;
  int o_heads, o_rows;  // head-split operand output (GemmLaunch::o_heads)
  // implicit-GEMM Conv2d: channels-last input [N][H][W][Cp] (or a zero-padded
  // [N][Hp][Wp][Cp] copy when Hp > 0), weight k = (kh*KWp + kw)*Cp + c
  const void* x_hi;
  const void* x_lo;
  int H, W, Cp, KH, KW, sh, sw, ph, pw, dh, dw, OH, OW;
  int Hp, Wp, KWp;
  // conv_tma: 0 = A rows gathered (CONV kernels) or a plain GEMM;
  // 1 = A boxes by TMA from the unpadded input, one (tap, 128 bytes of
  //     channels) per k-block; 2 = A windows by TMA from the padded input,
  //     one filter row per k-block.  Modes 1 and 2 tile the output as TH x TW
  //     pixels.  3 = halo-staged (conv_halo_kernel): output pixels numbered
  //     in the padded row space, halo_rows input rows per 128-byte channel
  //     block.
  int conv_tma, TW, TH, tiles_w, tiles_h;
  int nimg, halo_rows;
  // 3x3 / stride 2 max pool (padding pool_pad, 0 or 1) fused into a ReLU
  // convolution (gemm_kernel POOL): pooled [img][PH][PW][N] at py + img*py_sn
  // + ph*py_sh + pw*py_sw + n (fp32, or null), and the operand at the same
  // offsets of o_hi / o_lo (or null)
  float* py;
  long long py_sn, py_sh, py_sw;
  int PH, PW, pool_pad;
  int pool_kw;  // pooled columns per tile: 31 (64-column windowed tiles) or 30 (row runs)
  // Split tail: the last partial wave's tail_r tiles (tail_first on) are each
  // split along K into tail_s parts, part i taken by CTA i; the parts'
  // accumulators meet in tail_ws (one 128 x BN slot per CTA), and the part
  // that arrives last (tail_cnt, one counter per tile, left at 0) sums them in
  // part order and runs the epilogue.  tail_s == 0: round-robin whole tiles.
  int tail_s, tail_r, tail_first;
  float* tail_ws;
  unsigned* tail_cnt;
  // Global average pool of a TMA-fed convolution's output (tiles inside one
  // image) replacing c: the column sums of lane quarter q of row tile tm go
  // to gap[(tm*4 + q)*N + n], to be added up per image by a pool step.
  float* gap;
};

// Work item j of this CTA: a whole tile, or one part of a split tail tile
// (part >= 0); k-blocks [k0, k1).  False past the CTA's last item.
__device__ __forceinline__ bool work_at(const GemmParams& p, int ntiles, int t0, int ts, int j, int& tile, int& k0,
                                        int& k1, int& part) {
  part = -1;
  k0 = 0;
  k1 = p.nkb;
  if (p.tail_s == 0) {
    tile = t0 + j * ts;
    return tile < ntiles;
  }
  const int nfull = (p.tail_first - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  if (j < nfull) {
    tile = (int)blockIdx.x + j * (int)gridDim.x;
    return true;
  }
  const int item = (int)blockIdx.x;
  if (j > nfull || item >= p.tail_r * p.tail_s) return false;
  tile = p.tail_first + item / p.tail_s;
  part = item % p.tail_s;
  k0 = part * p.nkb / p.tail_s;
  k1 = (part + 1) * p.nkb / p.tail_s;
  return true;
}


// Store one 32-row x 16-column block of a tile.  `ep` holds it row-major
// with a 20-float row pitch; each pass a warp writes 8 rows x 16 columns,
// lane l taking row l/4 and columns 4*(l%4)..+3 (a float4 where the output
// is contiguous and aligned).  v = act(acc*sc[n] + sh[n]) (+ residual).
// Write 4 consecutive values of a row as operand elements (split or bf16).
template <int PREC>
__device__ __forceinline__ void store_operand4(void* ohi, float* olo, long long off, const float (&v)[4]) {
  if constexpr (PREC == PFC_PRECISION_BF16) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&a);
    pk.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(ohi) + off) = pk;
  } else {
    float4 h, l;
    split_tf32(v[0], h.x, l.x);
    split_tf32(v[1], h.y, l.y);
    split_tf32(v[2], h.z, l.z);
    split_tf32(v[3], h.w, l.w);
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(ohi) + off) = h;
    *reinterpret_cast<float4*>(olo + off) = l;
  }
}
template <int PREC>
__device__ __forceinline__ void store_operand1(void* ohi, float* olo, long long off, float v) {
  if constexpr (PREC == PFC_PRECISION_BF16) {
    reinterpret_cast<__nv_bfloat16*>(ohi)[off] = __float2bfloat16_rn(v);
  } else {
    float h, l;
    split_tf32(v, h, l);
    reinterpret_cast<float*>(ohi)[off] = h;
    olo[off] = l;
  }
}

// Output row of virtual row v of a halo-staged convolution (pixels numbered
// (img*Hp + oh)*Wp + ow in the padded row space), or -1 for a padding pixel.
// (The host keeps N*Hp*Wp + 128 below 2^31, so 32-bit division suffices.)
__device__ __forceinline__ long long halo_out_row(const GemmParams& p, long long v) {
  const unsigned hw = (unsigned)(p.Hp * p.Wp), vv = (unsigned)v;
  const unsigned img = vv / hw, rem = vv - img * hw;
  const unsigned oh = rem / (unsigned)p.Wp, ow = rem - oh * (unsigned)p.Wp;
  if (img >= (unsigned)p.nimg || oh >= (unsigned)p.OH || ow >= (unsigned)p.OW) return -1;
  return ((long long)img * p.OH + oh) * p.OW + ow;
}

// Element offset of operand output (row, n): row-major with pitch o_sm, or
// head-split [(b*heads + h)*rows + l][d] for row = b*rows + l, n = h*o_sm + d.
__device__ __forceinline__ long long op_offset(const GemmParams& p, long long row, int n) {
  if (p.o_heads == 0) return row * p.o_sm + n;
  const long long b = row / p.o_rows, l = row - b * p.o_rows;
  const int h = n / (int)p.o_sm, d = n - h * (int)p.o_sm;
  return ((b * p.o_heads + h) * p.o_rows + l) * p.o_sm + d;
}

// Rows m_base .. m_base+31 of the output matrix, of which the first nvalid
// exist; MAPPED: virtual rows m_base .. of a halo-staged convolution.
template <int ACT, int PREC, bool MAPPED = false>
__device__ __forceinline__ void store_block(const GemmParams& p, const float* ep, long long m_base, int nvalid, int n0,
                                            float* cbase, const float* rbase, void* ohi, float* olo, bool vec_c,
                                            bool vec_r, float alpha, float bsc, bool has_shift, int lane) {
  const int rsub = lane >> 2, c4 = (lane & 3) * 4;
  const int n = n0 + c4;
  float sc[4], sh[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sc[j] = alpha;
    sh[j] = bsc;
    if (n + j < p.N) {
      if (p.scale) { sc[j] = p.scale[n + j]; sh[j] = p.shift[n + j]; }
      else if (p.bias) sh[j] = p.bias[n + j];
    }
  }
  const bool full_n = n + 3 < p.N;
  // all four passes' shared-memory reads in flight at once
  float4 a[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) a[k] = *reinterpret_cast<const float4*>(ep + (8 * k + rsub) * 20 + c4);
  if (!MAPPED && full_n && vec_c && nvalid == 32 && !rbase) {
    // whole block inside the output, no residual: straight float4 stores
    const long long c0 = (m_base + rsub) * p.c_sm + n, cstep = 8 * p.c_sm;
    // (a head-split operand keeps 32-row blocks inside one batch: same step)
    const long long o0 = ohi ? op_offset(p, m_base + rsub, n) : 0, ostep = 8 * p.o_sm;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float v[4] = {a[k].x, a[k].y, a[k].z, a[k].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[j] = v[j] * sc[j];
        if (has_shift) v[j] = v[j] + sh[j];
        v[j] = act_apply<ACT>(v[j]);
      }
      if (cbase) *reinterpret_cast<float4*>(cbase + c0 + k * cstep) = make_float4(v[0], v[1], v[2], v[3]);
      if (ohi) store_operand4<PREC>(ohi, olo, o0 + k * ostep, v);
    }
    return;
  }
  if (!MAPPED && full_n && vec_c && vec_r && nvalid == 32 && rbase) {
    // whole block with a float4 residual: all four residual loads in flight
    // before the first store (one memory latency per block, not four)
    const long long c0 = (m_base + rsub) * p.c_sm + n, cstep = 8 * p.c_sm;
    const long long r0 = (m_base + rsub) * p.r_sm + n, rstep = 8 * p.r_sm;
    const long long o0 = ohi ? op_offset(p, m_base + rsub, n) : 0, ostep = 8 * p.o_sm;
    float4 r[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) r[k] = *reinterpret_cast<const float4*>(rbase + r0 + k * rstep);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float v[4] = {a[k].x, a[k].y, a[k].z, a[k].w};
      const float rr[4] = {r[k].x, r[k].y, r[k].z, r[k].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[j] = v[j] * sc[j];
        if (has_shift) v[j] = v[j] + sh[j];
        v[j] = act_apply<ACT>(v[j]) + rr[j];
      }
      if (cbase) *reinterpret_cast<float4*>(cbase + c0 + k * cstep) = make_float4(v[0], v[1], v[2], v[3]);
      if (ohi) store_operand4<PREC>(ohi, olo, o0 + k * ostep, v);
    }
    return;
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    long long row = m_base + 8 * k + rsub;
    if constexpr (MAPPED) row = halo_out_row(p, row);
    float v[4] = {a[k].x, a[k].y, a[k].z, a[k].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] = v[j] * sc[j];
      if (has_shift) v[j] = v[j] + sh[j];
      v[j] = act_apply<ACT>(v[j]);
    }
    if (MAPPED ? row < 0 : 8 * k + rsub >= nvalid) continue;
    const long long co = row * p.c_sm + (long long)n * p.c_sn;
    const long long oo = ohi ? op_offset(p, row, n) : 0;
    if (full_n && vec_c) {
      if (rbase) {
        const long long ro = row * p.r_sm + (long long)n * p.r_sn;
        if (vec_r) {
          const float4 r4 = *reinterpret_cast<const float4*>(rbase + ro);
          v[0] += r4.x; v[1] += r4.y; v[2] += r4.z; v[3] += r4.w;
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) v[j] += rbase[ro + (long long)j * p.r_sn];
        }
      }
      if (cbase) *reinterpret_cast<float4*>(cbase + co) = make_float4(v[0], v[1], v[2], v[3]);
      if (ohi) store_operand4<PREC>(ohi, olo, oo, v);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (n + j >= p.N) break;
        float w = v[j];
        if (rbase) w += rbase[row * p.r_sm + (long long)(n + j) * p.r_sn];
        if (cbase) cbase[co + (long long)j * p.c_sn] = w;
        if (ohi) store_operand1<PREC>(ohi, olo, oo + j, w);
      }
    }
  }
}

template <int PREC, int BN, bool CAT_ = false>
struct Cfg {
  static constexpr int ESZ = PREC == PFC_PRECISION_BF16 ? 2 : 4;
  static constexpr int BK = 128 / ESZ;  // K elements per 128-byte swizzle row
  static constexpr int UK = PREC == PFC_PRECISION_BF16 ? 16 : 8;
  static constexpr int KSTEPS = BK / UK;
  static constexpr int NOPS = PREC == PFC_PRECISION_BF16 ? 1 : 2;
  static constexpr int A_TILE = kBM * 128;
  static constexpr int B_TILE = BN * 128;
  static constexpr int STAGE = NOPS * (A_TILE + B_TILE);
  // stage layout [A_hi][A_lo][B_hi][B_lo]: B_hi and B_lo adjacent, so one
  // descriptor spans both as a 2*BN-row operand
  static constexpr int A_LO_OFF = A_TILE;
  static constexpr int B_HI_OFF = NOPS * A_TILE;
  static constexpr int B_LO_OFF = B_HI_OFF + B_TILE;
  // CAT (64-column 3xTF32 tiles): A_hi x [B_hi | B_lo] as ONE N = 128
  // instruction (64 cycles, against 2 x 48 for two N = 64 ones, and A_hi
  // read once instead of twice), then A_lo x B_hi (N = 64) into the first
  // half; the epilogue adds the two halves.  A separate kernel
  // instantiation, so the MMA issue loop carries no branch.
  static constexpr bool CAT = CAT_ && NOPS == 2 && BN == 64;
  static constexpr int ACC_COLS = CAT ? 2 * BN : BN;  // columns per accumulator
  // epilogue staging: per epilogue warp a 32 x 33 fp32 tile (padded: no bank conflicts)
  static constexpr int EPI_WARP_FLOATS = 32 * 20;  // a 32 x 16 block, 20-float pitch
  static constexpr int EPI_BYTES = kEpiWarps * EPI_WARP_FLOATS * 4;
  static constexpr int SMEM_LIMIT = 232448;  // 227 KB opt-in maximum per block
  static constexpr int STAGES_FIT = (SMEM_LIMIT - EPI_BYTES - 2048) / STAGE;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int SMEM = STAGES * STAGE + EPI_BYTES + 1024 /*barriers*/ + 1024 /*align*/;
  static constexpr int TMEM_COLS = 2 * ACC_COLS;  // two accumulators: epilogue of tile i overlaps MMAs of tile i+1
  static constexpr uint32_t IDESC = idesc(kBM, BN, PREC == PFC_PRECISION_BF16 ? 1u : 2u);
  static constexpr uint32_t IDESC_CAT = idesc(kBM, 2 * BN, 2u);
  static_assert(STAGES >= 2, "shared memory too small for two stages");
  static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM allocation");
};

// 16-byte global->shared copy; src_bytes 0 writes zeros (padding).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// make this thread's completed generic-proxy shared-memory writes visible to
// the tensor cores (async proxy)
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }


// Tile t of the persistent schedule -> (batch, m tile, n tile).  Within a
// batch slice, groups of 16 M-tiles sweep all N-tiles, so the B tiles of a
// group stay in L2 while the group's A rows stream.
__device__ __forceinline__ void tile_coords(const GemmParams& p, int t, int& bz, int& tm, int& tn) {
  const int per_batch = p.num_m * p.num_n;
  bz = t / per_batch;
  const int r = t - bz * per_batch;
  const int group = 16;
  const int per_group = group * p.num_n;
  const int first_m = (r / per_group) * group;
  const int gsz = min(p.num_m - first_m, group);
  tm = first_m + (r % per_group) % gsz;
  tn = (r % per_group) / gsz;
}

// Output tile tm of a TMA-fed convolution -> (image, first output row, first
// output column); the tile is TH x TW output pixels.
__device__ __forceinline__ void conv_tile(const GemmParams& p, int tm, int& img, int& oh0, int& ow0) {
  const int per_img = p.tiles_h * p.tiles_w;
  img = tm / per_img;
  const int r = tm - img * per_img;
  oh0 = (r / p.tiles_w) * p.TH;
  ow0 = (r % p.tiles_w) * p.TW;
}

// Tiles of a pool-fused convolution: strips of tiles_h tiles, one strip per
// (image, column tile colt), u = (img*tiles_w + colt)*tiles_h + pos.  With
// kw = pool_kw pooled columns per tile, tile (a, colt) is conv rows 2a, 2a+1
// and columns 2kw*colt-pad .. +63 (64 output pixels, TH = 2, TW = 64, of
// which the first 2kw+1 are used): pooled row a, columns kw*colt ..
// kw*colt+kw-1, with one more conv row carried from the tile walked before it
// in the strip.  Padding 1: row 2a-1, walking top-down (a = pos); padding 0:
// row 2a+2, walking bottom-up (a = tiles_h-1-pos).  The first tile of a strip
// carries a padding row.  pos is returned for that test.
__device__ __forceinline__ void pool_tile(const GemmParams& p, int u, int& img, int& oh0, int& ow0, int& a,
                                          int& colt, int& pos) {
  const int strip = u / p.tiles_h;
  pos = u - strip * p.tiles_h;
  img = strip / p.tiles_w;
  colt = strip - img * p.tiles_w;
  a = p.pool_pad ? pos : p.tiles_h - 1 - pos;
  oh0 = 2 * a;
  ow0 = 2 * p.pool_kw * colt - p.pool_pad;
}

// The CTA's run of consecutive tiles [own0, u1), so that each tile's carry
// comes from the tile before it; a run that starts inside a strip first
// recomputes the tile above (u0 = own0 - 1), for its carry only.
__device__ __forceinline__ void pool_run(const GemmParams& p, int ntiles, int& u0, int& u1, int& own0) {
  own0 = (int)((long long)blockIdx.x * ntiles / gridDim.x);
  u1 = (int)((long long)(blockIdx.x + 1) * ntiles / gridDim.x);
  u0 = (own0 < u1 && own0 % p.tiles_h != 0) ? own0 - 1 : own0;
}

// Barrier among the eight epilogue warps (named barrier 1) that also tells
// them whether any of them passed `v` true.
__device__ __forceinline__ bool epi_bar_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kEpiWarps * 32)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory"); }

// Column sums of v = act(acc*sc[n] + sh[n]) over this warp's first nvalid
// rows (lane = row) for columns n0 .. n0+HALF, written to slot[n]: each
// 32-column block is reduced across the lanes by halving exchanges (31
// shuffles, a fixed order), after which lane l holds column l's sum.
template <int ACT, int HALF>
__device__ __forceinline__ void gap_block(const GemmParams& p, const float (&acc)[HALF], int n0, int nvalid,
                                          float alpha, float bsc, bool has_shift, int lane, float* slot) {
#pragma unroll
  for (int cc = 0; cc < HALF; cc += 32) {
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = n0 + cc + j;
      float sc = alpha, sh = bsc;
      if (n < p.N) {
        if (p.scale) {
          sc = p.scale[n];
          sh = p.shift[n];
        } else if (p.bias) {
          sh = p.bias[n];
        }
      }
      float x = acc[cc + j] * sc;
      if (has_shift) x = x + sh;
      x = act_apply<ACT>(x);
      v[j] = lane < nvalid ? x : 0.f;  // a select: rows outside the image add nothing, NaN included
    }
#pragma unroll
    for (int w = 16; w >= 1; w >>= 1) {
      const bool up = (lane & w) != 0;
#pragma unroll
      for (int j = 0; j < w; ++j) {
        const float send = up ? v[j] : v[j + w];
        const float keep = up ? v[j + w] : v[j];
        v[j] = keep + __shfl_xor_sync(0xffffffffu, send, w);
      }
    }
    if (n0 + cc + lane < p.N) slot[n0 + cc + lane] = v[0];
  }
}

// Epilogue warp e (0..7) on TMEM lane quarter q: for every tile this CTA
// owns, sum the chunk accumulators in registers (handing each accumulator
// back to the MMA warp at once), then apply alpha/bias/folded-BN/activation/
// residual and store 32 x 16 blocks through this warp's staging area ep.
// rows(tm, m_base, nvalid) names the warp's 32 output rows.  GAP: column
// sums into GemmParams::gap instead of stores (activation 0 or 1 only).
template <int PREC, int BN, bool CAT, bool MAPPED, bool GAP, class Rows>
__device__ __forceinline__ void run_epilogue(const GemmParams& p, uint32_t tmem, uint64_t* acc_full,
                                             uint64_t* acc_empty, float* ep, int e, int q, int lane, Rows rows) {
  using C = Cfg<PREC, BN, CAT>;
  constexpr int HALF = BN / 2;  // columns per epilogue warp
  const int col0 = (e >> 2) * HALF;
  const int nkb = p.nkb;
  const int ntiles = p.num_m * p.num_n * p.batch;
  const float alpha = p.alpha_ptr ? *p.alpha_ptr : p.alpha;
  const float bsc = p.bias_scalar ? *p.bias_scalar : 0.f;
  const bool has_shift = p.scale || p.bias || p.bias_scalar;
  __shared__ int s_last;  // a split tail tile: this CTA's part arrived last
  int u = 0;
  bool ok = true;
  // With a split tail a warp whose wait failed keeps walking its items (no
  // more waits) so that every warp meets the split tile's barriers, where
  // all eight leave together; otherwise it leaves at once.
  for (int wj = 0; ok || (!MAPPED && p.tail_s); ++wj) {
    int t, k0, k1, part;
    if (!work_at(p, ntiles, blockIdx.x, gridDim.x, wj, t, k0, k1, part)) break;
    const int nch = k1 > k0 ? (k1 - k0 + p.kchunk - 1) / p.kchunk : 1;
    // this thread's row of the tile, columns col0..col0+HALF: the sum of the chunk accumulators
    float acc[HALF];
#pragma unroll
    for (int j = 0; j < HALF; ++j) acc[j] = 0.f;
    for (int ch = 0; ch < nch && ok; ++ch, ++u) {
      const int b = u & 1;
      const uint32_t use = (uint32_t)(u >> 1);
      // one outcome per warp: the TMEM loads below are warp-collective
      // (sleeping between tries: measured 1-4 % faster GEMMs than spinning)
      if (!__all_sync(0xffffffffu, mbar_wait_backoff(smem_u32(&acc_full[b]), use & 1u, p.err))) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (nkb > 0) {
#pragma unroll
        for (int cc = 0; cc < HALF; cc += 32) {
          uint32_t r[32];
          const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * C::ACC_COLS + col0 + cc);
          tmem_ld16_nowait(ta, *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
          tmem_ld16_nowait(ta + 16, *reinterpret_cast<uint32_t(*)[16]>(&r[16]));
          if constexpr (C::CAT) {
            // the A_hi x B_lo half of a concatenated accumulator
            uint32_t r2[32];
            tmem_ld16_nowait(ta + BN, *reinterpret_cast<uint32_t(*)[16]>(&r2[0]));
            tmem_ld16_nowait(ta + BN + 16, *reinterpret_cast<uint32_t(*)[16]>(&r2[16]));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[cc + j] += __uint_as_float(r[j]) + __uint_as_float(r2[j]);
          } else {
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[cc + j] += __uint_as_float(r[j]);
          }
        }
      }
      // the chunk is in registers: hand the accumulator back to the MMA warp
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&acc_empty[b]));
    }
    if (!MAPPED && part >= 0) {
      // a part of a split tail tile: its accumulator rows go to this CTA's
      // slot; the part that arrives last sums all parts in part order
      // (deterministic whichever CTA it is) and stores the tile
      float* slot = p.tail_ws + (size_t)blockIdx.x * (kBM * BN) + (size_t)(q * 32 + lane) * BN + col0;
#pragma unroll
      for (int j = 0; j < HALF; j += 4)
        *reinterpret_cast<float4*>(slot + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
      __threadfence();
      if (epi_bar_any(!ok)) break;
      if (e == 0 && lane == 0) {
        const unsigned prev = atomicAdd(&p.tail_cnt[t - p.tail_first], 1u);
        s_last = prev == (unsigned)(p.tail_s - 1);
        if (s_last) p.tail_cnt[t - p.tail_first] = 0u;  // ready for the next launch
      }
      epi_bar();
      if (!s_last) continue;
      __threadfence();  // the other parts' slots, written before their arrivals
      const int item0 = (t - p.tail_first) * p.tail_s;
#pragma unroll
      for (int j = 0; j < HALF; ++j) acc[j] = 0.f;
      for (int s2 = 0; s2 < p.tail_s; ++s2) {
        const float* src = p.tail_ws + (size_t)(item0 + s2) * (kBM * BN) + (size_t)(q * 32 + lane) * BN + col0;
#pragma unroll
        for (int j = 0; j < HALF; j += 4) {
          const float4 v4 = __ldcg(reinterpret_cast<const float4*>(src + j));
          acc[j] += v4.x;
          acc[j + 1] += v4.y;
          acc[j + 2] += v4.z;
          acc[j + 3] += v4.w;
        }
      }
    }
    if (!ok) {
      if (MAPPED || p.tail_s == 0) break;
      continue;
    }
    int bz, tm, tn;
    tile_coords(p, t, bz, tm, tn);
    const int n0 = tn * BN + col0;
    // this warp's 32 rows: output matrix rows m_base.., the first nvalid of which exist
    long long m_base;
    int nvalid;
    rows(tm, m_base, nvalid);
    if constexpr (GAP) {
      float* slot = p.gap + ((long long)tm * 4 + q) * p.N;
      if (p.act == 1) gap_block<1, HALF>(p, acc, n0, nvalid, alpha, bsc, has_shift, lane, slot);
      else gap_block<0, HALF>(p, acc, n0, nvalid, alpha, bsc, has_shift, lane, slot);
      continue;
    } else {
      float* cbase = p.c ? p.c + (long long)bz * p.c_sb : nullptr;
      const float* rbase = p.res ? p.res + (long long)bz * p.r_sb : nullptr;
      const long long obatch = (long long)bz * p.M * p.o_sm;
      void* ohi = p.o_hi ? (void*)((char*)p.o_hi + obatch * C::ESZ) : nullptr;
      float* olo = p.o_lo ? p.o_lo + obatch : nullptr;
      // float4 stores need contiguous, 16-byte aligned rows of the output (and residual)
      const bool vec_c = !cbase || (p.c_sn == 1 && (p.c_sm & 3) == 0 && (((uintptr_t)cbase) & 15) == 0);
      const bool vec_r = rbase && p.r_sn == 1 && (p.r_sm & 3) == 0 && (((uintptr_t)rbase) & 15) == 0;
#pragma unroll
      for (int cc = 0; cc < HALF; cc += 16) {
        // transpose through shared memory: this lane's row in, 8 rows x 16 columns out per pass
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          *reinterpret_cast<float4*>(ep + lane * 20 + j) = make_float4(acc[cc + j], acc[cc + j + 1], acc[cc + j + 2], acc[cc + j + 3]);
        __syncwarp();
        switch (p.act) {
          case 1: store_block<1, PREC, MAPPED>(p, ep, m_base, nvalid, n0 + cc, cbase, rbase, ohi, olo, vec_c, vec_r, alpha, bsc, has_shift, lane); break;
          case 2: store_block<2, PREC, MAPPED>(p, ep, m_base, nvalid, n0 + cc, cbase, rbase, ohi, olo, vec_c, vec_r, alpha, bsc, has_shift, lane); break;
          case 3: store_block<3, PREC, MAPPED>(p, ep, m_base, nvalid, n0 + cc, cbase, rbase, ohi, olo, vec_c, vec_r, alpha, bsc, has_shift, lane); break;
          case 4: store_block<4, PREC, MAPPED>(p, ep, m_base, nvalid, n0 + cc, cbase, rbase, ohi, olo, vec_c, vec_r, alpha, bsc, has_shift, lane); break;
          case 5: store_block<5, PREC, MAPPED>(p, ep, m_base, nvalid, n0 + cc, cbase, rbase, ohi, olo, vec_c, vec_r, alpha, bsc, has_shift, lane); break;
          default: store_block<0, PREC, MAPPED>(p, ep, m_base, nvalid, n0 + cc, cbase, rbase, ohi, olo, vec_c, vec_r, alpha, bsc, has_shift, lane); break;
        }
        __syncwarp();
      }
    }
  }
}

// Epilogue of a convolution with BN = N = 64 whose ReLU output feeds a 3x3 /
// stride 2 max pool (padding 0 or 1) and nothing else (PyFlame's Conv2d ->
// BatchNorm -> ReLU -> MaxPool2d stem): the conv output never reaches
// memory.  Thread (lane quarter q, lane) holds conv pixel (row r = q >> 1,
// column x = 32(q & 1) + lane) of the tile, channels 32(e >> 2) .. +31.
// Values are >= +0 after the ReLU and never NaN (ReLU maps NaN to 0), so the
// pool's max is exact in any order and pixels outside the image can enter it
// as 0: every window holds a real pixel.  Of the tile's two rows, row rc
// (1 for padding 1, 0 for padding 0) is the one the next tile of the strip
// needs; the other, ro, makes pooled row a with it and the carried row.  Per
// tile:
//   1. v = relu(acc*scale + shift) (0 outside the image); even columns take
//      the max of columns x, x+1, x+2 by shuffles (pooled column x/2).
//   2. Row rc writes its window maxima to the next-carry buffer; the pixels
//      of the one window that spans two warps (columns 30..32) go to shared
//      memory; barrier.
//   3. Row ro combines the carry, its own and row rc's maxima into pooled row
//      a and stores it as fp32 and / or the next convolution's operand; the
//      spanning window (pooled column 15) is finished by a warp of row rc,
//      whose other work is lighter, with a channel per lane.
// The eight epilogue warps meet at two named barriers per tile, so every
// warp takes every tile; a failed wait is agreed on at the first barrier.
// Scale and shift are staged per channel in shared memory once.  (Clock
// counters in a copy built outside the product put the epilogue, not the
// MMAs, on the critical path of the 7-k-block stem: 3.3K cycles per tile
// computing v with the scale and shift read from global memory, 2.9K in a
// single lane finishing column 15, against 4.8K cycles of MMA issue.)
template <int PREC, int BN, bool CAT>
__device__ __forceinline__ void run_pool_epilogue(const GemmParams& p, uint32_t tmem, uint64_t* acc_full,
                                                  uint64_t* acc_empty, float* sm, int e, int q, int lane, int u0,
                                                  int u1, int own0) {
  using C = Cfg<PREC, BN, CAT>;
  static_assert(BN == 64, "the pooled epilogue takes 64-channel tiles");
  static_assert((2 * 64 * 32 + 4 * 64 + 3 * 64) * 4 <= C::EPI_BYTES, "pool buffers exceed the epilogue staging area");
  constexpr int HALF = BN / 2;
  const int KW = p.pool_kw;  // pooled columns per tile (30 or 31; column 15 spans the warps)
  const int col0 = (e >> 2) * HALF;
  const int r = q >> 1, x = (q & 1) * 32 + lane, kq = x >> 1;
  const int rc = p.pool_pad ? 1 : 0, ro = 1 - rc;
  // window maxima of the carried conv row, [2][64 channels][32 pooled
  // columns]: lanes at consecutive pooled columns touch consecutive words
  // (no bank conflicts beside the tensor core's operand reads)
  float* rowbuf = sm;
  float* bnd = sm + 2 * 64 * 32;  // [4][64]: row ro column 32, row rc columns 30, 31, 32
  float2* scsh = reinterpret_cast<float2*>(sm + 2 * 64 * 32 + 4 * 64);  // [64] (scale, shift) per channel
  float* h30 = sm + 2 * 64 * 32 + 4 * 64 + 2 * 64;  // [64]: row ro's maxima of columns 30, 31
  // warp q = 2ro finishes pooled column 15 (conv columns 30..32 span two warps)
  // warp q = 2rc (of the lighter row) finishes pooled column 15 (conv
  // columns 30..32 span two warps), from lane 30 of warp q = 2ro
  const bool span = q == 2 * rc, ro30 = q == 2 * ro && lane == 30;
  const int bslot = q == 2 * ro + 1 && lane == 0 ? 0
                    : q == 2 * rc && lane == 30  ? 1
                    : q == 2 * rc && lane == 31  ? 2
                    : q == 2 * rc + 1 && lane == 0 ? 3
                                                   : -1;
  const float alpha = p.alpha_ptr ? *p.alpha_ptr : p.alpha;
  const float bsc = p.bias_scalar ? *p.bias_scalar : 0.f;
  const bool has_shift = p.scale || p.bias || p.bias_scalar;
  {
    // per-channel scale and shift once, in shared memory (visible after the
    // first tile's barrier): every tile reads them with broadcast loads
    const int i = e * 32 + lane;
    if (i < 64) {
      float sc = alpha, sh = bsc;
      if (p.scale) {
        sc = p.scale[i];
        sh = p.shift[i];
      } else if (p.bias) {
        sh = p.bias[i];
      }
      scsh[i] = make_float2(sc, sh);
    }
  }
  int u = 0;
  bool ok = true;
  for (int t = u0; t < u1; ++t) {
    float acc[HALF];
#pragma unroll
    for (int j = 0; j < HALF; ++j) acc[j] = 0.f;
    for (int ch = 0; ch < p.nchunks && ok; ++ch, ++u) {
      const int b = u & 1;
      const uint32_t use = (uint32_t)(u >> 1);
      if (!__all_sync(0xffffffffu, mbar_wait_backoff(smem_u32(&acc_full[b]), use & 1u, p.err))) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint32_t rr[32];
      const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * C::ACC_COLS + col0);
      tmem_ld16_nowait(ta, *reinterpret_cast<uint32_t(*)[16]>(&rr[0]));
      tmem_ld16_nowait(ta + 16, *reinterpret_cast<uint32_t(*)[16]>(&rr[16]));
      if constexpr (C::CAT) {
        // the A_hi x B_lo half of a concatenated accumulator
        uint32_t r2[32];
        tmem_ld16_nowait(ta + BN, *reinterpret_cast<uint32_t(*)[16]>(&r2[0]));
        tmem_ld16_nowait(ta + BN + 16, *reinterpret_cast<uint32_t(*)[16]>(&r2[16]));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] += __uint_as_float(rr[j]) + __uint_as_float(r2[j]);
      } else {
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] += __uint_as_float(rr[j]);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&acc_empty[b]));
    }
    // all warps leave together on a failed wait; otherwise the barrier after
    // which the previous tile's reads of the shared buffers are done
    if (epi_bar_any(!ok)) break;
    int img, oh0, ow0, a, colt, pos;
    pool_tile(p, t, img, oh0, ow0, a, colt, pos);
    const int oh = oh0 + r, ow = ow0 + x;
    // (tile columns past 2KW feed no window: row runs leave them unloaded)
    const bool real = oh < p.OH && ow >= 0 && ow < p.OW && x <= 2 * KW;
    float v[HALF], hm[HALF];
#pragma unroll
    for (int j = 0; j < HALF; ++j) {
      const float2 ss = scsh[col0 + j];
      float w = acc[j] * ss.x;
      if (has_shift) w = w + ss.y;
      w = act_apply<1>(w);
      v[j] = real ? w : 0.f;
    }
#pragma unroll
    for (int j = 0; j < HALF; ++j) {
      const float a1 = __shfl_down_sync(0xffffffffu, v[j], 1);
      const float a2 = __shfl_down_sync(0xffffffffu, v[j], 2);  // lanes 30, 31: their own value
      hm[j] = fmaxf(v[j], fmaxf(a1, a2));
    }
    float* next = rowbuf + (t & 1) * (64 * 32) + col0 * 32;  // this warp's channels
    const float* carry = rowbuf + ((t - 1) & 1) * (64 * 32) + col0 * 32;
    if (r == rc && (lane & 1) == 0 && kq < KW && kq != 15) {
#pragma unroll
      for (int j = 0; j < HALF; ++j) next[j * 32 + kq] = hm[j];
    }
    if (bslot >= 0) {
#pragma unroll
      for (int j = 0; j < HALF; j += 4)
        *reinterpret_cast<float4*>(bnd + bslot * 64 + col0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    }
    if (ro30) {
#pragma unroll
      for (int j = 0; j < HALF; j += 4)
        *reinterpret_cast<float4*>(h30 + col0 + j) = make_float4(hm[j], hm[j + 1], hm[j + 2], hm[j + 3]);
    }
    epi_bar();
    if (span) {
      // pooled column 15 with one channel per lane (n = col0 + lane): row
      // rc's window (its next carry) from the boundary pixels, row ro's from
      // its lane 30's maxima of columns 30, 31 and column 32
      const int n = col0 + lane;
      const float h1 = fmaxf(bnd[64 + n], fmaxf(bnd[128 + n], bnd[192 + n]));
      next[lane * 32 + 15] = h1;
      const int pw = KW * colt + 15;
      if (t >= own0 && 15 < KW && pw < p.PW && a < p.PH) {
        const float c = pos == 0 ? 0.f : carry[lane * 32 + 15];
        const float o = fmaxf(c, fmaxf(fmaxf(h30[n], bnd[n]), h1));
        const long long off = (long long)img * p.py_sn + (long long)a * p.py_sh + (long long)pw * p.py_sw + n;
        if (p.py) p.py[off] = o;
        if (p.o_hi) store_operand1<PREC>(p.o_hi, p.o_lo, off, o);
      }
    }
    // Row ro: pooled column kq of lane pair (2kq, 2kq+1), the even lane
    // taking channels 8i..8i+3 and the odd lane 8i+4..8i+7 (i = 0..3), so
    // that each store instruction writes whole 32-byte sectors; the odd lane
    // takes its window maxima from the even one.  (t, own0 and r are uniform
    // over the warp.)  The tile recomputed before a run only feeds the carry.
    if (r == ro && t >= own0) {
      const int odd = lane & 1;
      float hs[HALF / 2];
#pragma unroll
      for (int i = 0; i < HALF / 8; ++i) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float y = __shfl_sync(0xffffffffu, hm[8 * i + 4 + u], lane & ~1);
          hs[4 * i + u] = odd ? y : hm[8 * i + u];
        }
      }
      const int pw = KW * colt + kq;
      if (kq < KW && !(q == 2 * ro && kq == 15) && pw < p.PW && a < p.PH) {
        const long long off = (long long)img * p.py_sn + (long long)a * p.py_sh + (long long)pw * p.py_sw + col0;
#pragma unroll
        for (int i = 0; i < HALF / 8; ++i) {
          const int j0 = 8 * i + 4 * odd;
          float o[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float h1 = next[(j0 + u) * 32 + kq];
            const float c = pos == 0 ? 0.f : carry[(j0 + u) * 32 + kq];  // a strip's first tile carries padding
            o[u] = fmaxf(c, fmaxf(hs[4 * i + u], h1));
          }
          if (p.py) *reinterpret_cast<float4*>(p.py + off + j0) = make_float4(o[0], o[1], o[2], o[3]);
          if (p.o_hi) store_operand4<PREC>(p.o_hi, p.o_lo, off + j0, o);
        }
      }
    }
  }
}

// Epilogue forms of gemm_kernel (separate instantiations, so that each
// carries only its own code): stores; a 3x3 / stride 2 max pool; the column
// sums of a global average pool.
constexpr int kEpiStore = 0, kEpiMaxPool = 1, kEpiAvg = 2;

// Persistent kernel: each CTA walks tiles blockIdx.x, +gridDim.x, ...
// CONV: the A operand is gathered by four producer warps from a channels-last
// input (implicit-GEMM Conv2d) instead of loaded by TMA.  EPI kEpiMaxPool: a
// windowed TMA convolution (conv_tma 2) with the max pool fused into its
// epilogue; each CTA walks a run of consecutive tiles (pool_run).  kEpiAvg:
// a TMA-fed convolution whose epilogue writes column sums (GemmParams::gap).
template <int PREC, int BN, bool CONV, bool CAT, int EPI = kEpiStore>
__global__ void __launch_bounds__(kThreads<CONV>, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
                const GemmParams p) {
  using C = Cfg<PREC, BN, CAT>;
  constexpr bool POOL = EPI == kEpiMaxPool;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* epi = (float*)(smem + C::STAGES * C::STAGE);
  uint64_t* bars = (uint64_t*)(smem + C::STAGES * C::STAGE + C::EPI_BYTES);
  uint64_t* full = bars;                       // [STAGES] TMA -> MMA
  uint64_t* empty = bars + C::STAGES;          // [STAGES] MMA -> TMA
  uint64_t* acc_full = bars + 2 * C::STAGES;   // [2] MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;          // [2] epilogue -> MMA
  uint64_t* done = acc_empty + 2;              // all MMAs of this CTA retired
  uint32_t* tmem_slot = (uint32_t*)(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // an earlier CTA gave up: stop early (block-uniform decision)
  __shared__ int s_stop;
  if (threadIdx.x == 0) s_stop = *(volatile int*)p.err;
  __syncthreads();
  if (s_stop != 0) return;

  constexpr int PW = kProdWarps<CONV>;  // warp index of the MMA issuer
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      // CONV: the B copy's expect_tx arrival plus one arrival per gathering thread
      mbar_init(smem_u32(&full[s]), CONV ? 1 + 32 * PW : 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), kEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(smem_u32(done), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == PW) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  const int nkb = p.nkb;
  const int ntiles = p.num_m * p.num_n * p.batch;
  // this CTA's tiles: t0, t0 + ts, ... below t1
  int t0 = blockIdx.x, t1 = ntiles, ts = gridDim.x, own0 = 0;
  if constexpr (POOL) {
    pool_run(p, ntiles, t0, t1, own0);
    ts = 1;
  }
  if (CONV && warp < PW) {
    // ---------------- implicit-GEMM producer: thread r gathers A row r ----------------
    const int r = threadIdx.x;
    constexpr int CH = 16 / C::ESZ;  // K elements per 16-byte chunk
    constexpr int D = C::STAGES - 1 < 2 ? C::STAGES - 1 : 2;  // k-blocks in flight before signalling
    const int taps = p.KH * p.KW;
    const int ohw = p.OH * p.OW;
    int g = 0, pending = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      int bz, tm, tn;
      tile_coords(p, t, bz, tm, tn);
      const int n0 = tn * BN;
      const int m = tm * kBM + r;
      const bool mok = m < p.M;
      int ih0 = 0, iw0 = 0;
      long long img_base = 0;
      // a zero-padded input is addressed in padded coordinates (no border checks needed)
      const int XH = p.Hp > 0 ? p.Hp : p.H, XW = p.Hp > 0 ? p.Wp : p.W;
      if (mok) {
        const int img = m / ohw, rem = m - img * ohw;
        const int oh = rem / p.OW, ow = rem - oh * p.OW;
        ih0 = oh * p.sh - (p.Hp > 0 ? 0 : p.ph);
        iw0 = ow * p.sw - (p.Hp > 0 ? 0 : p.pw);
        img_base = (long long)img * XH * XW * p.Cp;
      }
      int c = 0, kw = 0, kh = 0, tap = 0;  // position of the next chunk along k
      for (int kb = 0; kb < nkb; ++kb, ++g) {
        const int s = g % C::STAGES;
        const uint32_t ph = (uint32_t)(g / C::STAGES) & 1u;
        if (g >= C::STAGES && !mbar_wait(smem_u32(&empty[s]), ph ^ 1u, p.err)) { ok = false; break; }
        uint8_t* st = smem + s * C::STAGE;
        if (r == 0) {
          const uint32_t fb = smem_u32(&full[s]);
          mbar_expect_tx(fb, C::NOPS * C::B_TILE);
          tma_load_3d(smem_u32(st + C::B_HI_OFF), &tb_hi, fb, kb * C::BK, n0, 0);
          if constexpr (C::NOPS == 2) tma_load_3d(smem_u32(st + C::B_LO_OFF), &tb_lo, fb, kb * C::BK, n0, 0);
        }
        const uint32_t arow_hi = smem_u32(st) + (uint32_t)r * 128u;
        const uint32_t arow_lo = smem_u32(st + C::A_LO_OFF) + (uint32_t)r * 128u;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int ih = ih0 + kh * p.dh, iw = iw0 + kw * p.dw;
          const bool in = mok && tap < taps && kw < p.KW && (unsigned)ih < (unsigned)XH && (unsigned)iw < (unsigned)XW;
          const long long off = in ? (img_base + ((long long)ih * XW + iw) * p.Cp + c) * C::ESZ : 0;
          const uint32_t sw = (uint32_t)((j ^ (r & 7)) << 4);  // 128-byte swizzle, as TMA writes it
          cp_async16(arow_hi + sw, (const char*)p.x_hi + off, in ? 16u : 0u);
          if constexpr (C::NOPS == 2) cp_async16(arow_lo + sw, (const char*)p.x_lo + off, in ? 16u : 0u);
          c += CH;
          if (c == p.Cp) {
            c = 0;
            if (++kw == p.KWp) { kw = 0; ++kh; }
            tap = kh * p.KW + kw;
          }
        }
        cp_async_commit();
        if (++pending > D) {
          cp_async_wait<D>();
          fence_proxy_async();
          mbar_arrive(smem_u32(&full[(g - D) % C::STAGES]));
          --pending;
        }
      }
    }
    cp_async_wait<0>();
    fence_proxy_async();
    for (int k = g - pending; k < g; ++k) mbar_arrive(smem_u32(&full[k % C::STAGES]));
    if (!ok && r == 0) {
      // an error stopped the pipeline: let this thread's B copies land before exit
      for (int k = g > C::STAGES ? g - C::STAGES : 0; k < g; ++k)
        mbar_wait_own(smem_u32(&full[k % C::STAGES]), (uint32_t)(k / C::STAGES) & 1u, p.err);
    }
  } else if (!CONV && warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    int g = 0;  // k-block counter across all tiles of this CTA
    bool ok = true;
    for (int wj = 0; ok; ++wj) {
      int t, k0, k1, part;
      if (!work_at(p, t1, t0, ts, wj, t, k0, k1, part)) break;
      int bz, tm, tn;
      tile_coords(p, t, bz, tm, tn);
      const int ca = p.a_batched ? bz : 0, cb = p.b_batched ? bz : 0;
      const int m0 = tm * kBM, n0 = tn * BN;
      for (int kb = k0; kb < k1; ++kb, ++g) {
        const int s = g % C::STAGES;
        const uint32_t ph = (uint32_t)(g / C::STAGES) & 1u;
        if (g >= C::STAGES && !mbar_wait(smem_u32(&empty[s]), ph ^ 1u, p.err)) { ok = false; break; }
        uint8_t* st = smem + s * C::STAGE;
        const uint32_t fb = smem_u32(&full[s]);
        mbar_expect_tx(fb, C::STAGE);
        const int kc = kb * C::BK;
        const uint32_t a_hi_dst = smem_u32(st), a_lo_dst = smem_u32(st + C::A_LO_OFF);
        if (p.conv_tma == 1) {
          // BK channels (128 bytes) of one filter tap: a TH x TW box of the input
          // shifted by the tap
          const int per_tap = p.Cp / C::BK;
          const int tap = kb / per_tap, c0 = (kb - tap * per_tap) * C::BK;
          const int kh = tap / p.KW, kw = tap - kh * p.KW;
          int img, oh0, ow0;
          conv_tile(p, tm, img, oh0, ow0);
          const int x0 = ow0 - p.pw + kw * p.dw, y0 = oh0 - p.ph + kh * p.dh;
          tma_load_4d(a_hi_dst, &ta_hi, fb, c0, x0, y0, img);
          if constexpr (C::NOPS == 2) tma_load_4d(a_lo_dst, &ta_lo, fb, c0, x0, y0, img);
        } else if (p.conv_tma == 2) {
          // filter row kb: for every output pixel a 128-byte window of the padded input
          int img, oh0, ow0;
          if constexpr (POOL) {
            int a, colt, pos;
            pool_tile(p, t, img, oh0, ow0, a, colt, pos);
          } else {
            conv_tile(p, tm, img, oh0, ow0);
          }
          tma_load_5d(a_hi_dst, &ta_hi, fb, 0, ow0, kb, oh0, img);
          if constexpr (C::NOPS == 2) tma_load_5d(a_lo_dst, &ta_lo, fb, 0, ow0, kb, oh0, img);
        } else {
          tma_load_3d(a_hi_dst, &ta_hi, fb, kc, m0, ca);
          if constexpr (C::NOPS == 2) tma_load_3d(a_lo_dst, &ta_lo, fb, kc, m0, ca);
        }
        tma_load_3d(smem_u32(st + C::B_HI_OFF), &tb_hi, fb, kc, n0, cb);
        if constexpr (C::NOPS == 2) tma_load_3d(smem_u32(st + C::B_LO_OFF), &tb_lo, fb, kc, n0, cb);
      }
    }
    // drain: every issued copy must have landed before the CTA can exit
    for (int k = g > C::STAGES ? g - C::STAGES : 0; k < g; ++k)
      mbar_wait_own(smem_u32(&full[k % C::STAGES]), (uint32_t)(k / C::STAGES) & 1u, p.err);
  } else if (warp == PW && lane == 0) {
    // ---------------- MMA issuer ----------------
    // K is accumulated in chunks of kchunk k-blocks, each into a fresh TMEM
    // accumulator (alternating between the two); the epilogue sums the chunks
    // in fp32 registers.  Short accumulation runs inside the tensor core keep
    // long contractions (K = 16384) within fp32-reference accuracy.
    int g = 0, u = 0;  // k-blocks consumed; accumulator uses
    bool ok = true;
    for (int wj = 0; ok; ++wj) {
      int t, k0, k1, part;
      if (!work_at(p, t1, t0, ts, wj, t, k0, k1, part)) break;
      const int nch = k1 > k0 ? (k1 - k0 + p.kchunk - 1) / p.kchunk : 1;
      for (int ch = 0; ch < nch && ok; ++ch, ++u) {
        const int b = u & 1;
        const uint32_t use = (uint32_t)(u >> 1);
        if (u >= 2 && !mbar_wait(smem_u32(&acc_empty[b]), (use & 1u) ^ 1u, p.err)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc_t = tmem + (uint32_t)(b * C::ACC_COLS);
        const int kb0 = k0 + ch * p.kchunk, kb1 = min(k1, kb0 + p.kchunk);
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int s = g % C::STAGES;
          const uint32_t ph = (uint32_t)(g / C::STAGES) & 1u;
          if (!mbar_wait(smem_u32(&full[s]), ph, p.err)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t st = smem_u32(smem + s * C::STAGE);
          const uint64_t da_hi = sdesc(st), db_hi = sdesc(st + C::B_HI_OFF);
          const uint64_t da_lo = sdesc(st + C::A_LO_OFF), db_lo = sdesc(st + C::B_LO_OFF);
#pragma unroll
          for (int ks = 0; ks < C::KSTEPS; ++ks) {
            const uint32_t koff = ks * 32;  // 32 bytes of K per instruction
            const uint32_t acc = (kb > kb0 || ks > 0) ? 1u : 0u;
            if constexpr (C::CAT) {
              // [A_hi B_hi | A_hi B_lo] (starts both halves), then + A_lo B_hi
              umma<PREC>(acc_t, desc_add(da_hi, koff), desc_add(db_hi, koff), C::IDESC_CAT, acc);
              umma<PREC>(acc_t, desc_add(da_lo, koff), desc_add(db_hi, koff), C::IDESC, 1u);
            } else if constexpr (C::NOPS == 2) {
              // small products first, then the leading term
              umma<PREC>(acc_t, desc_add(da_lo, koff), desc_add(db_hi, koff), C::IDESC, acc);
              umma<PREC>(acc_t, desc_add(da_hi, koff), desc_add(db_lo, koff), C::IDESC, 1u);
              umma<PREC>(acc_t, desc_add(da_hi, koff), desc_add(db_hi, koff), C::IDESC, 1u);
            } else {
              umma<PREC>(acc_t, desc_add(da_hi, koff), desc_add(db_hi, koff), C::IDESC, acc);
            }
          }
          umma_commit(smem_u32(&empty[s]));
        }
        if (ok) umma_commit(smem_u32(&acc_full[b]));
      }
    }
    // retire every MMA this thread issued before TMEM is released
    umma_commit(smem_u32(done));
  } else if (warp > PW) {
    // ---------------- epilogue ----------------
    const int e = warp - PW - 1;  // 0..7
    if constexpr (POOL) {
      run_pool_epilogue<PREC, BN, CAT>(p, tmem, acc_full, acc_empty, epi, e, warp & 3, lane, t0, t1, own0);
    } else
    run_epilogue<PREC, BN, CAT, false, EPI == kEpiAvg>(p, tmem, acc_full, acc_empty, epi + e * C::EPI_WARP_FLOATS, e,
                                                   warp & 3, lane,
                                  [&](int tm, long long& m_base, int& nvalid) {
                                    const int q = warp & 3;
                                    if (p.conv_tma) {
                                      int img, oh0, ow0;
                                      conv_tile(p, tm, img, oh0, ow0);
                                      // TW >= 32: the warp's rows lie in one output row
                                      const int oh = oh0 + (q * 32) / p.TW, ow = ow0 + (q * 32) % p.TW;
                                      m_base = ((long long)img * p.OH + oh) * p.OW + ow;
                                      nvalid = oh < p.OH ? max(0, min(32, p.OW - ow)) : 0;
                                    } else {
                                      m_base = (long long)tm * kBM + q * 32;
                                      nvalid = max(0, min(32, p.M - (int)m_base));
                                    }
                                  });
  }
  // teardown: wait until every MMA of this CTA retired, then release TMEM
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == PW) {
    if (lane == 0) mbar_wait_own(smem_u32(done), 0u, p.err);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// The pooled stem over row runs.
//
// A stride-2 convolution whose filter row is one k-block of 8 taps of
// 16-byte pixels (tf32: 4 channels, bf16: 8), over a zero-padded input whose
// rows hold their even columns first, then their odd columns ([N][Hp][2]
// [Wp/2][16 bytes], ConvInputLaunch::deint).  At stride 2, taps 2i and 2i+1
// of output column ow read even and odd column ow + i: so the 64 output
// columns of a tile read, from each padded input row, a run of 64 even and a
// run of 64 odd pixels (1 KB each), and the A operand of k-step i is that
// pair of runs entered i pixels later.  That is a K-major operand without
// swizzle: 8 pixels x 16 bytes per core matrix (rows 16 bytes apart, 8-row
// groups 128 bytes apart), the odd run LBO bytes after the even one.
// The tile's conv rows oh and oh+1 read padded rows 2oh + kh and 2oh + kh + 2.
// Its KH + 2 input rows are stored in the order 0, 2, 4, .., 1, 3, .., 1 KB
// apart, so row 2oh+kh+2 directly follows row 2oh+kh and MMA rows 64..127
// (conv row oh+1) continue rows 0..63 (conv row oh) with the same group
// stride.  Output columns 61..63 of each conv row read into the following
// run and feed no pooled window: a tile covers 61 columns, 30 pooled ones.
// Per tile the input crosses L2 once (36 KB for tf32x3, against 7 x 32 KB of
// overlapping TMA windows), and the filter stays in shared memory.
// Warps: 0 loads the filter once, then each tile's runs (1-D bulk copies)
// into NA buffers; 1 issues the MMAs; 2..9 run the pooled epilogue.
template <int PREC, bool CAT>
struct RowsCfg {
  using G = Cfg<PREC, 64, CAT>;
  static constexpr int RUN = 64 * 16;                // one run: 64 pixels of 16 bytes
  static constexpr int MAXKH = 7;
  static constexpr int SLOTS = MAXKH + 2;            // input rows per tile
  static constexpr int A_OP = 2 * SLOTS * RUN;       // per operand: even runs, then odd runs
  static constexpr int A_BUF = G::NOPS * A_OP;
  static constexpr int B_KB = G::NOPS * G::B_TILE;   // one filter row, [B_hi | B_lo]
  static constexpr int B_BYTES = MAXKH * B_KB;
  static constexpr int NA_FIT = (G::SMEM_LIMIT - 1024 - B_BYTES - G::EPI_BYTES - 2048) / A_BUF;
  static constexpr int NA = NA_FIT > 4 ? 4 : NA_FIT;
  static constexpr int SMEM = B_BYTES + NA * A_BUF + G::EPI_BYTES + 1024 /*barriers*/ + 1024 /*align*/;
  static_assert(NA >= 2, "shared memory too small for two run buffers");
  static_assert(G::KSTEPS == 4, "a k-block is 8 taps of 16-byte pixels");
};

template <int PREC, bool CAT>
__global__ void __launch_bounds__(kThreads<false>, 1)
    conv_rows_pool_kernel(const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
                          const GemmParams p) {
  using C = Cfg<PREC, 64, CAT>;
  using R = RowsCfg<PREC, CAT>;
  constexpr int NA = R::NA;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* bres = smem;                              // [KH][B_hi | B_lo]
  uint8_t* abuf = smem + R::B_BYTES;                 // [NA][NOPS][even runs | odd runs]
  float* epi = (float*)(abuf + NA * R::A_BUF);
  uint64_t* bfull = (uint64_t*)((uint8_t*)epi + C::EPI_BYTES);  // filter landed
  uint64_t* afull = bfull + 1;                                  // [NA] runs landed
  uint64_t* aempty = afull + NA;                                // [NA] runs consumed
  uint64_t* acc_full = aempty + NA;                             // [2] MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;                           // [2] epilogue -> MMA
  uint64_t* done = acc_empty + 2;                               // all MMAs retired
  uint32_t* tmem_slot = (uint32_t*)(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int s_stop;
  if (threadIdx.x == 0) s_stop = *(volatile int*)p.err;
  __syncthreads();
  if (s_stop != 0) return;

  constexpr int PW = 1;  // MMA warp
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(bfull), 1);
    for (int s = 0; s < NA; ++s) {
      mbar_init(smem_u32(&afull[s]), 1);
      mbar_init(smem_u32(&aempty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), kEpiWarps);
    }
    mbar_init(smem_u32(done), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == PW) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  int u0, u1, own0;
  pool_run(p, p.num_m, u0, u1, own0);
  const int KH = p.KH, nev = (KH + 3) / 2;  // input rows 0..KH+1; nev of them even
  if (warp == 0 && lane == 0) {
    // ---------------- producer: the filter once, then each tile's runs ----------------
    const uint32_t bb = smem_u32(bfull);
    mbar_expect_tx(bb, (uint32_t)(KH * R::B_KB));
    for (int kh = 0; kh < KH; ++kh) {
      tma_load_3d(smem_u32(bres + kh * R::B_KB), &tb_hi, bb, kh * C::BK, 0, 0);
      if constexpr (C::NOPS == 2) tma_load_3d(smem_u32(bres + kh * R::B_KB + C::B_TILE), &tb_lo, bb, kh * C::BK, 0, 0);
    }
    const int half = p.Wp / 2;  // pixels per run of a padded row
    const uint8_t* xh = (const uint8_t*)p.x_hi;
    const uint8_t* xl = (const uint8_t*)p.x_lo;
    int g = 0;
    for (int t = u0; t < u1; ++t, ++g) {
      const int s = g % NA;
      const uint32_t ph = (uint32_t)(g / NA) & 1u;
      if (g >= NA && !mbar_wait(smem_u32(&aempty[s]), ph ^ 1u, p.err)) break;
      int img, oh0, ow0, a, colt, pos;
      pool_tile(p, t, img, oh0, ow0, a, colt, pos);
      // pixels [ow0, ow0 + 64) of each run, clipped to the row; input rows
      // past the padded image feed only conv rows past OH
      const int e0 = max(ow0, 0), e1 = min(ow0 + 64, half);
      const int r0 = 2 * oh0, nr = min(KH + 2, p.Hp - r0);
      const uint32_t bytes = e1 > e0 ? (uint32_t)(e1 - e0) * 16u : 0u;
      uint8_t* dst = abuf + s * R::A_BUF;
      const uint32_t fb = smem_u32(&afull[s]);
      mbar_expect_tx(fb, bytes * (uint32_t)(2 * nr * C::NOPS));
      if (bytes == 0) continue;
      for (int r = 0; r < nr; ++r) {
        const int slot = (r & 1) ? nev + (r >> 1) : (r >> 1);
        const long long rowpix = ((long long)img * p.Hp + r0 + r) * p.Wp;
        for (int par = 0; par < 2; ++par) {
          const long long src = (rowpix + (long long)par * half + e0) * 16;
          const uint32_t off = (uint32_t)((par * R::SLOTS + slot) * R::RUN + (e0 - ow0) * 16);
          bulk_g2s(smem_u32(dst + off), xh + src, bytes, fb);
          if constexpr (C::NOPS == 2) bulk_g2s(smem_u32(dst + R::A_OP + off), xl + src, bytes, fb);
        }
      }
    }
    // every issued copy must have landed before the CTA can exit
    mbar_wait_own(bb, 0u, p.err);
    for (int k = g > NA ? g - NA : 0; k < g; ++k)
      mbar_wait_own(smem_u32(&afull[k % NA]), (uint32_t)(k / NA) & 1u, p.err);
  } else if (warp == PW && lane == 0) {
    // ---------------- MMA issuer ----------------
    bool ok = mbar_wait(smem_u32(bfull), 0u, p.err);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t a_base = smem_u32(abuf), b_base = smem_u32(bres);
    int g = 0;
    for (int t = u0; t < u1 && ok; ++t, ++g) {
      const int b = g & 1;
      const uint32_t use = (uint32_t)(g >> 1);
      if (g >= 2 && !mbar_wait(smem_u32(&acc_empty[b]), (use & 1u) ^ 1u, p.err)) break;
      const int s = g % NA;
      if (!mbar_wait(smem_u32(&afull[s]), (uint32_t)(g / NA) & 1u, p.err)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t acc_t = tmem + (uint32_t)(b * C::ACC_COLS);
      const uint32_t ab = a_base + (uint32_t)(s * R::A_BUF);
      for (int kh = 0; kh < KH; ++kh) {
        const int slot = (kh & 1) ? nev + (kh >> 1) : (kh >> 1);
        const uint64_t da_hi = sdesc_kint(ab + (uint32_t)(slot * R::RUN), R::SLOTS * R::RUN, 128);
        const uint64_t da_lo = desc_add(da_hi, R::A_OP);
        const uint64_t db_hi = sdesc(b_base + (uint32_t)(kh * R::B_KB));
        const uint64_t db_lo = desc_add(db_hi, C::B_TILE);
#pragma unroll
        for (int ks = 0; ks < C::KSTEPS; ++ks) {
          const uint32_t aoff = ks * 16, koff = ks * 32;  // one pixel further along both runs; 32 bytes of K
          const uint32_t acc = (kh > 0 || ks > 0) ? 1u : 0u;
          if constexpr (C::CAT) {
            umma<PREC>(acc_t, desc_add(da_hi, aoff), desc_add(db_hi, koff), C::IDESC_CAT, acc);
            umma<PREC>(acc_t, desc_add(da_lo, aoff), desc_add(db_hi, koff), C::IDESC, 1u);
          } else if constexpr (C::NOPS == 2) {
            umma<PREC>(acc_t, desc_add(da_lo, aoff), desc_add(db_hi, koff), C::IDESC, acc);
            umma<PREC>(acc_t, desc_add(da_hi, aoff), desc_add(db_lo, koff), C::IDESC, 1u);
            umma<PREC>(acc_t, desc_add(da_hi, aoff), desc_add(db_hi, koff), C::IDESC, 1u);
          } else {
            umma<PREC>(acc_t, desc_add(da_hi, aoff), desc_add(db_hi, koff), C::IDESC, acc);
          }
        }
      }
      umma_commit(smem_u32(&aempty[s]));
      umma_commit(smem_u32(&acc_full[b]));
    }
    umma_commit(smem_u32(done));
  } else if (warp > PW) {
    run_pool_epilogue<PREC, 64, CAT>(p, tmem, acc_full, acc_empty, epi, warp - PW - 1, warp & 3, lane, u0, u1, own0);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == PW) {
    if (lane == 0) mbar_wait_own(smem_u32(done), 0u, p.err);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// Halo-staged implicit-GEMM convolution (stride 1).
//
// The input is the zero-padded channels-last copy [N][Hp][Wp][Cp], seen as
// N*Hp*Wp rows of Cp channels.  Output pixels are numbered in the same row
// space, v = (img*Hp + oh)*Wp + ow; pixels with ow >= OW or oh >= OH are
// computed and dropped.  At stride 1 tap (kh, kw) of pixel v reads input row
// v + kh*dh*Wp + kw*dw, so the 128 pixels of a tile need one contiguous run of
// 128 + (KH-1)*dh*Wp + (KW-1)*dw input rows: the halo.  One TMA copy brings
// the halo of a 32-channel block into shared memory, and the A operand of
// every tap is the same run entered kh*dh*Wp + kw*dw rows later, so the input
// crosses L2 once per channel block instead of once per tap.
// Warps: 0 streams B (one tap x channel block per stage), 1 allocates TMEM and
// issues the MMAs, 2..9 run the epilogue, 10 loads halos into two buffers.
template <int PREC, int BN>
struct HaloCfg {
  using G = Cfg<PREC, BN>;  // the stage layout and sizes do not depend on CAT
  static constexpr int HROWS = 256;  // halo rows per buffer (one TMA box)
  static constexpr int H_OP = HROWS * 128;
  static constexpr int H_BUF = G::NOPS * H_OP;
  static constexpr int B_STAGE = G::NOPS * G::B_TILE;
  static constexpr int B_FIT = (G::SMEM_LIMIT - G::EPI_BYTES - 2048 - 2 * H_BUF) / B_STAGE;
  static constexpr int B_STAGES = B_FIT > 8 ? 8 : B_FIT;
  static constexpr int SMEM = 2 * H_BUF + B_STAGES * B_STAGE + G::EPI_BYTES + 1024 /*barriers*/ + 1024 /*align*/;
  static_assert(B_STAGES >= 2, "shared memory too small for the halo kernel");
};
constexpr int kHaloThreads = (1 + 1 + kEpiWarps + 1) * 32;

template <int PREC, int BN, bool CAT>
__global__ void __launch_bounds__(kHaloThreads, 1)
    conv_halo_kernel(const __grid_constant__ CUtensorMap tx_hi, const __grid_constant__ CUtensorMap tx_lo,
                     const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
                     const GemmParams p) {
  using C = Cfg<PREC, BN, CAT>;
  using H = HaloCfg<PREC, BN>;
  constexpr int S = H::B_STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* halo = smem;                    // [2][NOPS][HROWS x 128 B]
  uint8_t* bst = smem + 2 * H::H_BUF;      // [S][NOPS][BN x 128 B]
  float* epi = (float*)(bst + S * H::B_STAGE);
  uint64_t* full = (uint64_t*)((uint8_t*)epi + C::EPI_BYTES);  // [S] B copy landed
  uint64_t* empty = full + S;                                  // [S] B stage consumed
  uint64_t* hfull = empty + S;                                 // [2] halo landed
  uint64_t* hempty = hfull + 2;                                // [2] halo consumed
  uint64_t* acc_full = hempty + 2;                             // [2] MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;                          // [2] epilogue -> MMA
  uint64_t* done = acc_empty + 2;                              // all MMAs retired
  uint32_t* tmem_slot = (uint32_t*)(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int s_stop;
  if (threadIdx.x == 0) s_stop = *(volatile int*)p.err;
  __syncthreads();
  if (s_stop != 0) return;

  constexpr int PW = 1;  // MMA warp
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&hfull[b]), 1);
      mbar_init(smem_u32(&hempty[b]), 1);
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), kEpiWarps);
    }
    mbar_init(smem_u32(done), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == PW) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  const int ntiles = p.num_m * p.num_n;
  const int ncb = p.Cp / C::BK, taps = p.KH * p.KW;
  if (warp == 0 && lane == 0) {
    // ---------------- B producer: weight columns (kh*KW + kw)*Cp + BK*cb ----------------
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      int bz, tm, tn;
      tile_coords(p, t, bz, tm, tn);
      const int n0 = tn * BN;
      for (int cb = 0; cb < ncb && ok; ++cb) {
        for (int tap = 0; tap < taps; ++tap, ++g) {
          const int s = g % S;
          const uint32_t ph = (uint32_t)(g / S) & 1u;
          if (g >= S && !mbar_wait(smem_u32(&empty[s]), ph ^ 1u, p.err)) { ok = false; break; }
          uint8_t* st = bst + s * H::B_STAGE;
          const uint32_t fb = smem_u32(&full[s]);
          mbar_expect_tx(fb, H::B_STAGE);
          const int kc = tap * p.Cp + cb * C::BK;
          tma_load_3d(smem_u32(st), &tb_hi, fb, kc, n0, 0);
          if constexpr (C::NOPS == 2) tma_load_3d(smem_u32(st + C::B_TILE), &tb_lo, fb, kc, n0, 0);
        }
      }
    }
    for (int k = g > S ? g - S : 0; k < g; ++k)
      mbar_wait_own(smem_u32(&full[k % S]), (uint32_t)(k / S) & 1u, p.err);
  } else if (warp == PW + 1 + kEpiWarps && lane == 0) {
    // ---------------- halo producer ----------------
    int h = 0;
    bool ok = true;
    const uint32_t bytes = (uint32_t)p.halo_rows * 128u * C::NOPS;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      int bz, tm, tn;
      tile_coords(p, t, bz, tm, tn);
      for (int cb = 0; cb < ncb; ++cb, ++h) {
        const int hb = h & 1;
        const uint32_t ph = (uint32_t)(h >> 1) & 1u;
        if (h >= 2 && !mbar_wait(smem_u32(&hempty[hb]), ph ^ 1u, p.err)) { ok = false; break; }
        uint8_t* dst = halo + hb * H::H_BUF;
        const uint32_t fb = smem_u32(&hfull[hb]);
        mbar_expect_tx(fb, bytes);
        tma_load_2d(smem_u32(dst), &tx_hi, fb, cb * C::BK, tm * kBM);
        if constexpr (C::NOPS == 2) tma_load_2d(smem_u32(dst + H::H_OP), &tx_lo, fb, cb * C::BK, tm * kBM);
      }
    }
    for (int k = h > 2 ? h - 2 : 0; k < h; ++k)
      mbar_wait_own(smem_u32(&hfull[k & 1]), (uint32_t)(k >> 1) & 1u, p.err);
  } else if (warp == PW && lane == 0) {
    // ---------------- MMA issuer ----------------
    // k-blocks run channel block by channel block, tap by tap within one;
    // every kchunk k-blocks of a tile go to a fresh accumulator.
    // The issuing thread keeps its per-k-block work to counters and additions:
    // any latency here stalls the tensor core.
    int h = 0, u = 0, s = 0;
    uint32_t sph = 0;  // phase parity of ring stage s
    const uint32_t row_step = (uint32_t)(p.dh * p.Wp) * 128u, col_step = (uint32_t)p.dw * 128u;
    const uint32_t b_base = smem_u32(bst);
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      int left = 0, j = 0, b = 0;  // k-blocks left in the current accumulation chunk
      uint32_t acc_t = tmem;
      for (int cb = 0; cb < ncb && ok; ++cb, ++h) {
        const int hb = h & 1;
        if (!mbar_wait(smem_u32(&hfull[hb]), (uint32_t)(h >> 1) & 1u, p.err)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t x_hi = smem_u32(halo + hb * H::H_BUF);
        uint32_t arow = 0;
        for (int kh = 0; kh < p.KH && ok; ++kh, arow += row_step) {
          uint32_t aoff = arow;
          for (int kw = 0; kw < p.KW; ++kw, aoff += col_step) {
            const bool first = left == 0;
            if (first) {
              b = u & 1;
              if (u >= 2 && !mbar_wait(smem_u32(&acc_empty[b]), (uint32_t)((u >> 1) & 1) ^ 1u, p.err)) {
                ok = false;
                break;
              }
              asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
              acc_t = tmem + (uint32_t)(b * C::ACC_COLS);
              left = min(p.kchunk, p.nkb - j);
            }
            if (!mbar_wait(smem_u32(&full[s]), sph, p.err)) { ok = false; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint64_t da_hi = sdesc(x_hi + aoff), da_lo = desc_add(da_hi, H::H_OP);
            const uint64_t db_hi = sdesc(b_base + (uint32_t)s * H::B_STAGE), db_lo = desc_add(db_hi, C::B_TILE);
#pragma unroll
            for (int ks = 0; ks < C::KSTEPS; ++ks) {
              const uint32_t koff = ks * 32;
              const uint32_t acc = (!first || ks > 0) ? 1u : 0u;
              if constexpr (C::CAT) {
                // [B_hi | B_lo] are adjacent in the stage: one N = 128 instruction
                umma<PREC>(acc_t, desc_add(da_hi, koff), desc_add(db_hi, koff), C::IDESC_CAT, acc);
                umma<PREC>(acc_t, desc_add(da_lo, koff), desc_add(db_hi, koff), C::IDESC, 1u);
              } else if constexpr (C::NOPS == 2) {
                umma<PREC>(acc_t, desc_add(da_lo, koff), desc_add(db_hi, koff), C::IDESC, acc);
                umma<PREC>(acc_t, desc_add(da_hi, koff), desc_add(db_lo, koff), C::IDESC, 1u);
                umma<PREC>(acc_t, desc_add(da_hi, koff), desc_add(db_hi, koff), C::IDESC, 1u);
              } else {
                umma<PREC>(acc_t, desc_add(da_hi, koff), desc_add(db_hi, koff), C::IDESC, acc);
              }
            }
            umma_commit(smem_u32(&empty[s]));
            if (++s == S) { s = 0; sph ^= 1u; }
            ++j;
            if (--left == 0) {
              umma_commit(smem_u32(&acc_full[b]));
              ++u;
            }
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(&hempty[hb]));
      }
    }
    umma_commit(smem_u32(done));
  } else if (warp > PW && warp <= PW + kEpiWarps) {
    // ---------------- epilogue ----------------
    const int e = warp - PW - 1;
    run_epilogue<PREC, BN, CAT, true, false>(p, tmem, acc_full, acc_empty, epi + e * C::EPI_WARP_FLOATS, e, warp & 3,
                                             lane,
                                 [&](int tm, long long& m_base, int& nvalid) {
                                   m_base = (long long)tm * kBM + (warp & 3) * 32;  // virtual rows
                                   nvalid = -1;
                                 });
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == PW) {
    if (lane == 0) mbar_wait_own(smem_u32(done), 0u, p.err);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
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

// A-operand maps of a TMA-fed convolution (box of TW x TH output pixels).
// Mode 1: the unpadded input [N][H][W][Cp], box (128 bytes of channels, TW, TH, 1).
// Mode 2: overlapping windows of the padded input [N][Hp][Wp][Cp]: dims
// (window of 128 bytes, output column at stride sw*Cp, filter row at dh
// padded input rows, output row at sh padded rows, image), box
// (window, TW, 1, TH, 1).  False when the driver rejects the map.
bool make_conv_map(const GemmLaunch& L, int prec, int mode, int TW, int TH, const void* base, CUtensorMap* m) {
  std::memset(m, 0, sizeof *m);
  const int esz = prec == PFC_PRECISION_BF16 ? 2 : 4;
  const CUtensorMapDataType dt = prec == PFC_PRECISION_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const cuuint64_t C = (cuuint64_t)L.Cp;
  CUresult r;
  if (mode == 1) {
    cuuint64_t dims[4] = {C, (cuuint64_t)L.W, (cuuint64_t)L.H, (cuuint64_t)L.batch_images};
    cuuint64_t strides[3] = {C * esz, C * L.W * esz, C * L.W * L.H * esz};
    cuuint32_t box[4] = {(cuuint32_t)(128 / esz), (cuuint32_t)TW, (cuuint32_t)TH, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    r = get_encode()(m, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    const cuuint64_t row = C * L.Wp * esz;  // bytes of one padded input row
    cuuint64_t dims[5] = {(cuuint64_t)(128 / esz), (cuuint64_t)L.OW, (cuuint64_t)L.KH, (cuuint64_t)L.OH,
                          (cuuint64_t)L.batch_images};
    cuuint64_t strides[4] = {(cuuint64_t)(L.sw * C * esz), row * L.dh, row * L.sh, row * L.Hp};
    cuuint32_t box[5] = {(cuuint32_t)(128 / esz), (cuuint32_t)TW, 1, (cuuint32_t)TH, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    r = get_encode()(m, dt, 5, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  return r == CUDA_SUCCESS;
}

// Input rows one halo-staged tile reads: 128 pixels plus the reach of the
// filter in the padded row space, rounded up to whole 8-row swizzle groups.
int64_t halo_rows(const GemmLaunch& L) {
  const int64_t reach = (L.KH - 1) * L.dh * L.Wp + (L.KW - 1) * L.dw;
  return (kBM + reach + 7) / 8 * 8;
}

// Mode 3: the padded input [N][Hp][Wp][Cp] as N*Hp*Wp rows, box (32
// channels, halo rows).  Rows past the end read as zero.
bool make_halo_map(const GemmLaunch& L, int prec, const void* base, CUtensorMap* m) {
  std::memset(m, 0, sizeof *m);
  const int esz = prec == PFC_PRECISION_BF16 ? 2 : 4;
  const CUtensorMapDataType dt = prec == PFC_PRECISION_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  cuuint64_t dims[2] = {(cuuint64_t)L.Cp, (cuuint64_t)(L.batch_images * L.Hp * L.Wp)};
  cuuint64_t strides[1] = {(cuuint64_t)(L.Cp * esz)};
  cuuint32_t box[2] = {(cuuint32_t)(128 / esz), (cuuint32_t)halo_rows(L)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode()(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int PREC, int BN, bool CONV>
void launch_t(const GemmLaunch& L, cudaStream_t stream, int conv_tma = 0, const CUtensorMap* conv_maps = nullptr,
              int TW = 0) {
  using C = Cfg<PREC, BN>;
  // per-device set-up once, safe when several host threads launch at once
  static std::once_flag attr_once[64];
  const int dev = current_device();
  std::call_once(attr_once[dev], [] {
    PFB_CUDA(cudaFuncSetAttribute(gemm_kernel<PREC, BN, CONV, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    if constexpr (Cfg<PREC, BN, true>::CAT)
      PFB_CUDA(cudaFuncSetAttribute(gemm_kernel<PREC, BN, CONV, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    C::SMEM));
    if constexpr (!CONV && BN == 64) {
      PFB_CUDA(cudaFuncSetAttribute(conv_rows_pool_kernel<PREC, Cfg<PREC, BN, true>::CAT>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    RowsCfg<PREC, Cfg<PREC, BN, true>::CAT>::SMEM));
      PFB_CUDA(cudaFuncSetAttribute(gemm_kernel<PREC, BN, false, false, kEpiMaxPool>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
      if constexpr (Cfg<PREC, BN, true>::CAT)
        PFB_CUDA(cudaFuncSetAttribute(gemm_kernel<PREC, BN, false, true, kEpiMaxPool>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    }
    if constexpr (!CONV) {
      PFB_CUDA(cudaFuncSetAttribute(gemm_kernel<PREC, BN, false, false, kEpiAvg>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
      if constexpr (Cfg<PREC, BN, true>::CAT)
        PFB_CUDA(cudaFuncSetAttribute(gemm_kernel<PREC, BN, false, true, kEpiAvg>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    }
    if constexpr (!CONV) {
      PFB_CUDA(cudaFuncSetAttribute(conv_halo_kernel<PREC, BN, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    HaloCfg<PREC, BN>::SMEM));
      if constexpr (Cfg<PREC, BN, true>::CAT)
        PFB_CUDA(cudaFuncSetAttribute(conv_halo_kernel<PREC, BN, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      HaloCfg<PREC, BN>::SMEM));
    }
  });
  const int64_t a_rows = L.M, b_rows = L.N;
  CUtensorMap tb_hi = make_map(L.b_hi, PREC, L.kpad, b_rows, L.b_sb ? L.batch : 1, BN);
  CUtensorMap tb_lo = PREC == PFC_PRECISION_BF16 ? tb_hi : make_map(L.b_lo, PREC, L.kpad, b_rows, L.b_sb ? L.batch : 1, BN);
  // CONV gathers A itself (its maps are unused); TMA-fed convolutions bring their own maps
  CUtensorMap ta_hi, ta_lo;
  if (conv_tma) {
    ta_hi = conv_maps[0];
    ta_lo = conv_maps[1];
  } else {
    ta_hi = CONV ? tb_hi : make_map(L.a_hi, PREC, L.kpad, a_rows, L.a_sb ? L.batch : 1, kBM);
    ta_lo = CONV || PREC == PFC_PRECISION_BF16 ? ta_hi
                                               : make_map(L.a_lo, PREC, L.kpad, a_rows, L.a_sb ? L.batch : 1, kBM);
  }
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
  p.batch = (int)L.batch;
  p.o_hi = L.out_hi;
  p.o_lo = L.out_lo;
  p.o_sm = L.o_sm;
  p.o_heads = (int)L.o_heads;
  p.o_rows = (int)L.o_rows;
  p.x_hi = L.x_hi;
  p.x_lo = L.x_lo;
  p.H = (int)L.H; p.W = (int)L.W; p.Cp = (int)L.Cp; p.KH = (int)L.KH; p.KW = (int)L.KW;
  p.sh = (int)L.sh; p.sw = (int)L.sw; p.ph = (int)L.ph; p.pw = (int)L.pw; p.dh = (int)L.dh; p.dw = (int)L.dw;
  p.OH = (int)L.OH; p.OW = (int)L.OW;
  p.Hp = (int)L.Hp; p.Wp = (int)L.Wp; p.KWp = (int)(L.KWp > 0 ? L.KWp : L.KW);
  p.conv_tma = conv_tma;
  p.TW = TW > 0 ? TW : 128;
  p.TH = 128 / p.TW;
  p.tiles_w = conv_tma ? (int)ceil_div(L.OW, p.TW) : 1;
  p.tiles_h = conv_tma ? (int)ceil_div(L.OH, p.TH) : 1;
  if (conv_tma) p.num_m = (int)(L.batch_images * p.tiles_h * p.tiles_w);
  p.nimg = (int)L.batch_images;
  p.halo_rows = 0;
  if (conv_tma == 3) {
    // halo-staged: tiles of 128 pixels of the padded row space
    p.num_m = (int)ceil_div(L.batch_images * L.Hp * L.Wp, kBM);
    p.halo_rows = (int)halo_rows(L);
    p.batch = 1;
  }
  if (L.K == 0) p.nkb = 0;
  p.py = L.pool_y;
  p.py_sn = L.pool_sn;
  p.py_sh = L.pool_sh;
  p.py_sw = L.pool_sw;
  p.PH = (int)L.PH;
  p.PW = (int)L.PW;
  p.pool_pad = L.pool_pad;
  p.gap = L.gap;
  if (L.gap) {
    // slots of an image: 4 per row tile, tiles_h x tiles_w row tiles
    PFB_CHECK_ARG((conv_tma == 1 || conv_tma == 2) && !L.pool && p.tiles_h * p.tiles_w * 4 == conv_gap_slots(L.OH, L.OW),
                  "gemm: a fused global average pool needs a TMA-fed convolution tiled inside each image");
  }
  p.pool_kw = 31;
  if (L.pool) {
    // pooled rows by conv row pairs; 31 pooled columns per 64-pixel tile of
    // windows, 30 per tile of row runs
    if (L.deint) {
      const int64_t esz = PREC == PFC_PRECISION_BF16 ? 2 : 4;
      PFB_CHECK_ARG(BN == 64 && L.N == 64 && L.Cp * esz == 16 && p.KWp * L.Cp == C::BK && L.K == L.KH * C::BK &&
                        L.sh == 2 && L.sw == 2 && L.dh == 1 && L.dw == 1 && L.KH >= 1 && L.KH <= 7 && L.Wp % 2 == 0 &&
                        L.Wp / 2 >= L.OW + 3 && L.batch_images * L.Hp * L.Wp < (1ll << 40),
                    "gemm: the row-run stem needs a stride-2 convolution of 8-tap, 16-byte-pixel filter rows over a "
                    "de-interleaved padded input");
      p.pool_kw = 30;
    } else {
      PFB_CHECK_ARG(conv_tma == 2 && p.TW == 64 && BN == 64 && L.N == 64, "gemm: the fused max pool needs the windowed "
                    "TMA convolution with 64 output channels");
    }
    p.tiles_h = (int)ceil_div(L.OH, 2);
    p.tiles_w = (int)ceil_div(L.PW, p.pool_kw);
    p.num_m = (int)(L.batch_images * p.tiles_h * p.tiles_w);
  }
  // The concatenated-B instantiation (Cfg::CAT) where a tile has enough
  // k-blocks that the MMAs, not the epilogue, set the pace: it doubles the
  // epilogue's TMEM reads, which a 7-k-block tile with the full store
  // epilogue (the 7x7 stem convolution) does not hide (measured 0.96 -> 1.20
  // ms), while 18-k-block tiles gain (3x3 convolutions, 0.54 -> 0.45 ms).
  // The pooled stem, whose epilogue stores a quarter of its tile, takes it
  // regardless (0.97 -> 0.94 ms).
  const bool cat = Cfg<PREC, BN, true>::CAT && p.nkb >= 12;
  // accumulation chunks of 512 elements of K (16 tf32 / 8 bf16 k-blocks)
  p.kchunk = 512 / C::BK;
  p.nchunks = p.nkb > 0 ? (p.nkb + p.kchunk - 1) / p.kchunk : 1;
  const int64_t ntiles = (int64_t)p.num_m * p.num_n * L.batch;
  PFB_CHECK_ARG(ntiles < (1ll << 31), "gemm: too many tiles");
  // persistent: one CTA per SM (the shared-memory ring admits one), never more CTAs than tiles
  const unsigned grid = (unsigned)std::min<int64_t>(ntiles, device_sm_count(dev));
  // Split tail: a last wave of r < grid tiles keeps r SMs busy for a whole
  // tile while the rest idle; instead each of those tiles is split along K
  // into s = grid / r parts, one per CTA.  Only where every part keeps at
  // least 16 k-blocks (K >= 512 per part): shorter parts measured slower
  // than the whole tile (768-deep GEMMs lost 15-20 us each, 3072-deep ones
  // gained 24 us).  Plain GEMMs only (the convolution feeds walk their own
  // schedules).
  p.tail_s = p.tail_r = p.tail_first = 0;
  p.tail_ws = L.tail_ws;
  p.tail_cnt = L.tail_cnt;
  if (!CONV && !conv_tma && !L.pool && L.tail_ws && L.tail_cnt && ntiles > grid) {
    const int64_t r = ntiles % grid;
    const int64_t sp = r > 0 ? std::min<int64_t>(grid / r, p.nkb / 16) : 0;
    if (sp >= 2 && r <= L.tail_cnt_len && (int64_t)grid * kBM * BN * 4 <= L.tail_ws_bytes) {
      p.tail_s = (int)sp;
      p.tail_r = (int)r;
      p.tail_first = (int)(ntiles - r);
    }
  }
  if constexpr (!CONV) {
    if (conv_tma == 3) {
      if constexpr (Cfg<PREC, BN, true>::CAT) {
        if (cat) {
          conv_halo_kernel<PREC, BN, true><<<grid, kHaloThreads, HaloCfg<PREC, BN>::SMEM, stream>>>(ta_hi, ta_lo, tb_hi,
                                                                                         tb_lo, p);
          PFB_CUDA(cudaGetLastError());
          return;
        }
      }
      conv_halo_kernel<PREC, BN, false><<<grid, kHaloThreads, HaloCfg<PREC, BN>::SMEM, stream>>>(ta_hi, ta_lo, tb_hi,
                                                                                         tb_lo, p);
      PFB_CUDA(cudaGetLastError());
      return;
    }
  }
  if constexpr (!CONV && BN == 64) {
    if (L.pool && L.deint) {
      if constexpr (Cfg<PREC, BN, true>::CAT) {
        conv_rows_pool_kernel<PREC, true><<<grid, kThreads<false>, RowsCfg<PREC, true>::SMEM, stream>>>(tb_hi, tb_lo, p);
      } else {
        conv_rows_pool_kernel<PREC, false><<<grid, kThreads<false>, RowsCfg<PREC, false>::SMEM, stream>>>(tb_hi, tb_lo,
                                                                                                         p);
      }
      PFB_CUDA(cudaGetLastError());
      return;
    }
    if (L.pool) {
      // the pooled stem takes the concatenated-B MMAs (its epilogue stores a
      // quarter of the tile, which leaves room for the doubled TMEM reads)
      if constexpr (Cfg<PREC, BN, true>::CAT) {
        gemm_kernel<PREC, BN, false, true, kEpiMaxPool><<<grid, kThreads<false>, C::SMEM, stream>>>(ta_hi, ta_lo, tb_hi,
                                                                                                   tb_lo, p);
        PFB_CUDA(cudaGetLastError());
        return;
      }
      gemm_kernel<PREC, BN, false, false, kEpiMaxPool><<<grid, kThreads<false>, C::SMEM, stream>>>(ta_hi, ta_lo, tb_hi,
                                                                                                  tb_lo, p);
      PFB_CUDA(cudaGetLastError());
      return;
    }
  }
  PFB_CHECK_ARG(!L.pool, "gemm: the fused max pool needs the windowed TMA convolution");
  if constexpr (!CONV) {
    if (L.gap) {
      if constexpr (Cfg<PREC, BN, true>::CAT) {
        if (cat) {
          gemm_kernel<PREC, BN, false, true, kEpiAvg><<<grid, kThreads<false>, C::SMEM, stream>>>(ta_hi, ta_lo, tb_hi,
                                                                                                 tb_lo, p);
          PFB_CUDA(cudaGetLastError());
          return;
        }
      }
      gemm_kernel<PREC, BN, false, false, kEpiAvg><<<grid, kThreads<false>, C::SMEM, stream>>>(ta_hi, ta_lo, tb_hi,
                                                                                              tb_lo, p);
      PFB_CUDA(cudaGetLastError());
      return;
    }
  }
  PFB_CHECK_ARG(!L.gap, "gemm: the fused global average pool needs a TMA-fed convolution");
  if constexpr (Cfg<PREC, BN, true>::CAT) {
    if (cat) {
      gemm_kernel<PREC, BN, CONV, true><<<grid, kThreads<CONV>, C::SMEM, stream>>>(ta_hi, ta_lo, tb_hi, tb_lo, p);
      PFB_CUDA(cudaGetLastError());
      return;
    }
  }
  gemm_kernel<PREC, BN, CONV, false><<<grid, kThreads<CONV>, C::SMEM, stream>>>(ta_hi, ta_lo, tb_hi, tb_lo, p);
  PFB_CUDA(cudaGetLastError());
}

}  // namespace

// 3-D operand map [batch][rows][kpad], box (128 bytes of K) x box_rows x 1,
// for the other tensor-core kernels.  mn32: the 128-byte swizzle with 32-byte
// atoms, the shared-memory layout tcgen05 reads an MN-major tf32 operand from.
CUtensorMap make_operand_map(const void* base, int prec, int64_t kpad, int64_t rows, int64_t batch, int box_rows,
                             bool mn32) {
  if (!mn32) return make_map(base, prec, kpad, rows, batch, box_rows);
  CUtensorMap m;
  std::memset(&m, 0, sizeof m);
  cuuint64_t dims[3] = {(cuuint64_t)kpad, (cuuint64_t)rows, (cuuint64_t)std::max<int64_t>(batch, 1)};
  cuuint64_t strides[2] = {(cuuint64_t)(kpad * 4), (cuuint64_t)(kpad * rows * 4)};
  cuuint32_t box[3] = {32, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  PFB_CHECK_ARG(prec == PFC_PRECISION_TF32X3, "MN-major operand maps are tf32 only");
  CUresult r = get_encode()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(PFC_ERR_CUDA, "cuTensorMapEncodeTiled (32-byte atoms) failed: " + std::to_string((int)r));
  return m;
}

// Which A feed a convolution can use: 1 or 2 (TMA, maps built) or 0 (gather).
int conv_tma_mode(const GemmLaunch& L, int prec, CUtensorMap* maps, int* TW) {
  if (!L.allow_tma_conv) return 0;
  const int esz = prec == PFC_PRECISION_BF16 ? 2 : 4;
  const int64_t bk = 128 / esz, kwp = L.KWp > 0 ? L.KWp : L.KW;
  // halo-staged: stride 1 over a padded input, whole 32-channel blocks, a
  // halo that fits one TMA box
  if (L.Hp > 0 && L.sh == 1 && L.sw == 1 && L.Cp % bk == 0 && kwp == L.KW &&
      halo_rows(L) <= HaloCfg<PFC_PRECISION_TF32X3, 64>::HROWS &&
      L.batch_images * L.Hp * L.Wp < (int64_t)INT32_MAX - 2 * kBM) {
    if (make_halo_map(L, prec, L.x_hi, &maps[0])) {
      if (prec == PFC_PRECISION_BF16) { maps[1] = maps[0]; return 3; }
      if (make_halo_map(L, prec, L.x_lo, &maps[1])) return 3;
    }
  }
  if (L.OW < 32) return 0;
  *TW = conv_tile_w(L.OW);
  int mode = 0;
  if (L.Hp == 0 && L.Cp % bk == 0 && L.sh == 1 && L.sw == 1 && kwp == L.KW) mode = 1;
  else if (L.Hp > 0 && kwp * L.Cp == bk && L.dw == 1 && (L.sw * L.Cp * esz) % 16 == 0) mode = 2;
  if (!mode) return 0;
  if (!make_conv_map(L, prec, mode, *TW, 128 / *TW, L.x_hi, &maps[0])) return 0;
  if (prec == PFC_PRECISION_BF16) maps[1] = maps[0];
  else if (!make_conv_map(L, prec, mode, *TW, 128 / *TW, L.x_lo, &maps[1])) return 0;
  return mode;
}

void launch_gemm(const GemmLaunch& L, cudaStream_t stream) {
  PFB_CHECK_ARG(L.M > 0 && L.N > 0 && L.batch > 0, "gemm: empty problem");
  PFB_CHECK_ARG(L.M < (1ll << 31) && L.N < (1ll << 31), "gemm: dimension too large");
  PFB_CHECK_ARG(L.err != nullptr, "gemm: error flag pointer required");
  PFB_CHECK_ARG(L.c || L.out_hi || L.pool_y || L.gap, "gemm: no output");
  if (L.gap) {
    PFB_CHECK_ARG(L.conv && !L.pool && !L.residual && L.batch == 1 && !L.c && !L.out_hi && L.OW >= 32 &&
                      (L.act == 0 || L.act == 1),
                  "gemm: a fused global average pool replaces the output of a convolution with rows of 32+ pixels "
                  "(no activation or ReLU)");
  }
  if (L.pool) {
    PFB_CHECK_ARG(L.conv && L.N == 64 && L.act == 1 && !L.residual && L.batch == 1 && L.Hp > 0 && L.PH > 0 &&
                      L.PW > 0 && (L.pool_pad == 0 || L.pool_pad == 1) &&
                      L.PH == (L.OH + 2 * L.pool_pad - 3) / 2 + 1 && L.PW == (L.OW + 2 * L.pool_pad - 3) / 2 + 1 &&
                      L.OW > 32,
                  "gemm: a fused max pool needs a ReLU convolution with 64 output channels over a padded input");
    PFB_CHECK_ARG(L.pool_sw % 4 == 0 && L.pool_sh % 4 == 0 && L.pool_sn % 4 == 0 &&
                      (((uintptr_t)L.pool_y | (uintptr_t)L.out_hi | (uintptr_t)L.out_lo) & 15) == 0 &&
                      (L.pool_y || L.out_hi) && (!L.out_hi || L.precision == PFC_PRECISION_BF16 || L.out_lo),
                  "gemm: the pooled output needs 16-byte aligned channels-last rows");
  }
  if (L.out_hi && L.o_heads > 0) {
    PFB_CHECK_ARG(L.batch == 1 && L.o_sm % 16 == 0 && L.o_heads * L.o_sm == L.N && L.o_rows % 32 == 0 &&
                      L.M % L.o_rows == 0 && !L.conv,
                  "gemm: head-split operand output needs 16-column heads, 32-row groups and batch 1");
  }
  if (L.out_hi && !L.pool) {
    PFB_CHECK_ARG(L.N % 4 == 0 && L.o_sm % 4 == 0 && (L.o_heads > 0 || L.o_sm >= L.N) && ((uintptr_t)L.out_hi & 15) == 0 &&
                      (L.precision == PFC_PRECISION_BF16 || (L.out_lo && ((uintptr_t)L.out_lo & 15) == 0)),
                  "gemm: operand output needs 16-byte aligned rows of a multiple of 4 columns");
  }
  const int64_t kal = L.precision == PFC_PRECISION_BF16 ? 64 : 32;
  PFB_CHECK_ARG(L.kpad % kal == 0 && L.kpad >= L.K, "gemm: kpad must be a multiple of the K tile and >= K");
  if (L.conv) {
    const int64_t ch = L.precision == PFC_PRECISION_BF16 ? 8 : 4;  // elements per 16-byte chunk
    PFB_CHECK_ARG(L.batch == 1 && L.a_sb == 0 && L.b_sb == 0, "conv gemm: no batch slices");
    PFB_CHECK_ARG(L.x_hi && ((uintptr_t)L.x_hi & 15) == 0 && (L.precision == PFC_PRECISION_BF16 ||
                                                               (L.x_lo && ((uintptr_t)L.x_lo & 15) == 0)),
                  "conv gemm: channels-last input must be 16-byte aligned");
    const int64_t kwp = L.KWp > 0 ? L.KWp : L.KW;
    PFB_CHECK_ARG(L.Cp > 0 && L.Cp % ch == 0 && kwp >= L.KW && L.K == L.KH * kwp * L.Cp, "conv gemm: bad channel padding");
    PFB_CHECK_ARG(L.Hp == 0 || (L.Hp >= (L.OH - 1) * L.sh + (L.KH - 1) * L.dh + 1 &&
                                L.Wp >= (L.OW - 1) * L.sw + (kwp - 1) * L.dw + 1),
                  "conv gemm: padded input too small");
    PFB_CHECK_ARG(L.M == L.M / (L.OH * L.OW) * L.OH * L.OW && L.H * L.W * L.Cp < (1ll << 40) &&
                      L.OH * L.OW < (1ll << 31) && L.KH * L.KW < (1 << 20),
                  "conv gemm: bad geometry");
  } else {
    PFB_CHECK_ARG(((uintptr_t)L.a_hi & 15) == 0, "gemm: operands must be 16-byte aligned");
  }
  PFB_CHECK_ARG(((uintptr_t)L.b_hi & 15) == 0, "gemm: operands must be 16-byte aligned");
  if (L.precision == PFC_PRECISION_BF16) {
    if (L.conv) {
      CUtensorMap maps[2];
      int TW = 0;
      const int mode = conv_tma_mode(L, PFC_PRECISION_BF16, maps, &TW);
      if (mode == 1 && L.N >= 128) launch_t<PFC_PRECISION_BF16, 128, false>(L, stream, mode, maps, TW);
      else if (mode) launch_t<PFC_PRECISION_BF16, 64, false>(L, stream, mode, maps, TW);
      else launch_t<PFC_PRECISION_BF16, 64, true>(L, stream);
    } else {
      if (L.N > 64) launch_t<PFC_PRECISION_BF16, 128, false>(L, stream);
      else launch_t<PFC_PRECISION_BF16, 64, false>(L, stream);
    }
  } else {
    PFB_CHECK_ARG(L.b_lo && (L.conv || L.a_lo), "gemm: tf32x3 needs lo operands");
    if (L.conv) {
      CUtensorMap maps[2];
      int TW = 0;
      const int mode = conv_tma_mode(L, PFC_PRECISION_TF32X3, maps, &TW);
      // TMA boxes (mode 1) with 128+ output channels take 128-column tiles: at
      // 64 columns an MMA costs the tensor core about as much as at 128
      // (measured 111 -> 188 TFLOP/s on 3x3 convolutions of 64 -> 128 channels)
      if (mode == 1 && L.N >= 128) launch_t<PFC_PRECISION_TF32X3, 128, false>(L, stream, mode, maps, TW);
      else if (mode) launch_t<PFC_PRECISION_TF32X3, 64, false>(L, stream, mode, maps, TW);
      // 64-column tiles: the gathering warps leave too few registers for a
      // 128-column accumulator (wider convolutions take several column tiles)
      else launch_t<PFC_PRECISION_TF32X3, 64, true>(L, stream);
    } else {
      if (L.N > 64) launch_t<PFC_PRECISION_TF32X3, 128, false>(L, stream);
      else launch_t<PFC_PRECISION_TF32X3, 64, false>(L, stream);
    }
  }
}

}  // namespace pfb
