// small_gemm.cu — Linear layers of small batches on the CUDA cores, and a
// two-layer perceptron (Linear, activation, Linear, optional softmax) in one
// launch.
//
// With M <= 256 rows a tensor-core GEMM has at most two 128-row tiles per
// output column block: a 64-row batch through Linear 784->256 keeps 2 of 148
// SMs busy for the whole K loop, and the chain Linear -> ReLU -> Linear ->
// softmax costs four launches whose latency dwarfs the 26 MFLOP of work.
// Here every warp of a grid that covers the device computes a 4 x 4 block of
// outputs, its 32 lanes splitting K (float4 loads, coalesced along the
// weight rows), and reduces the 16 partial sums with shuffles; the bias,
// scale and activation are applied by the lane that holds each result.  For
// two layers, the CTA that finishes layer 1 last (an arrival counter zeroed
// before the launch; no CTA waits on another) computes layer 2 from the
// layer-1 rows in L2 and then the row softmax, so the whole chain is one
// launch with no grid-wide barrier.  Products accumulate in fp32 FMAs, in a
// different order than PyFlame's sequential sums (matmul.cpp:12-31): within
// a few ulp times sqrt(K) of them.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "../common.hpp"
#include "act.cuh"
#include "kernels.hpp"
#include "tcgen05.cuh"

namespace pfb {

namespace {

constexpr int kSWarps = 8;  // warps per CTA

struct SLayer {
  const float* w;  // weight rows W[n][k] (Linear's [out, in] weight), row pitch ldw
  long long ldw;
  const float* bias;  // bias[n * bstride] or null
  long long bstride;
  float alpha;
  const float* alpha_ptr;
  int N, K, act;
  int vec;  // float4 loads along K
};

struct SParams {
  const float* a;
  long long lda;
  int M;
  SLayer l1, l2;
  int layers;
  float* h;  // layer-1 rows when layers == 2
  long long ldh;
  float* out;
  long long ldo;
  int softmax;  // 0 none, 1 softmax, 2 log-softmax over the last layer's row
  unsigned long long* counter;
  int l2_smem;  // layer 2 from shared-memory copies of h and w2 (dynamic shared memory)
};

constexpr size_t kSmallSmemMax = 160 * 1024;  // largest staging of layer 2

// Loads by source: 0 global read-only (__ldg), 1 global through L2 (data
// written earlier in this launch by other CTAs), 2 shared memory.
template <int SRC>
__device__ __forceinline__ float4 ld4(const float* p) {
  if constexpr (SRC == 1) return __ldcg(reinterpret_cast<const float4*>(p));
  else if constexpr (SRC == 2) return *reinterpret_cast<const float4*>(p);
  else return __ldg(reinterpret_cast<const float4*>(p));
}
template <int SRC>
__device__ __forceinline__ float ld1(const float* p) {
  if constexpr (SRC == 1) return __ldcg(p);
  else if constexpr (SRC == 2) return *p;
  else return __ldg(p);
}

// Warp `wid` of `nwarps`: 4 x 4 output blocks of act(alpha * x W^T + bias)
// for the M rows of x (pitch ldx), written to dst[m * ldd + n].  XS / WS:
// where x and the weight rows are read from (ld4 / ld1 sources).
template <bool VEC, int XS, int WS>
__device__ void layer_tiles(const float* x, long long ldx, int M, const SLayer& L, float* dst, long long ldd, int wid,
                            int nwarps, int lane) {
  const int tm = (M + 3) >> 2, tn = (L.N + 3) >> 2;
  const float alpha = L.alpha_ptr ? *L.alpha_ptr : L.alpha;
  for (int t = wid; t < tm * tn; t += nwarps) {
    const int m0 = (t / tn) * 4, n0 = (t % tn) * 4;
    const float* xr[4];
    const float* wr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xr[i] = x + (long long)min(m0 + i, M - 1) * ldx;  // rows past the end repeat the last (not stored)
      wr[i] = L.w + (long long)min(n0 + i, L.N - 1) * L.ldw;
    }
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    if constexpr (VEC) {
#pragma unroll 2
      for (int k = lane * 4; k < L.K; k += 128) {
        float4 xa[4], wb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          xa[i] = ld4<XS>(xr[i] + k);
          wb[i] = ld4<WS>(wr[i] + k);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            acc[i][j] = fmaf(xa[i].x, wb[j].x, acc[i][j]);
            acc[i][j] = fmaf(xa[i].y, wb[j].y, acc[i][j]);
            acc[i][j] = fmaf(xa[i].z, wb[j].z, acc[i][j]);
            acc[i][j] = fmaf(xa[i].w, wb[j].w, acc[i][j]);
          }
      }
    } else {
      for (int k = lane; k < L.K; k += 32) {
        float xa[4], wb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          xa[i] = ld1<XS>(xr[i] + k);
          wb[i] = ld1<WS>(wr[i] + k);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wb[j], acc[i][j]);
      }
    }
    float mine = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float v = acc[i][j];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == i * 4 + j) mine = v;
      }
    if (lane < 16) {
      const int m = m0 + (lane >> 2), n = n0 + (lane & 3);
      if (m < M && n < L.N) {
        float v = mine * alpha;
        if (L.bias) v += L.bias[(long long)n * L.bstride];
        dst[(long long)m * ldd + n] = act_apply_rt(L.act, v);
      }
    }
  }
}

// The same for short rows (K <= kShortK): warp `wid` takes 4 rows x 32
// columns, lane = column; each lane runs the K loop over its weight row
// (float4) against the 4 rows of x, which all lanes read at the same address
// (one broadcast transaction).  No cross-lane reduction; no idle lanes when K
// is shorter than a warp's 128-element stride.
template <bool VEC>
__device__ void layer_rows32(const float* x, long long ldx, int M, const SLayer& L, float* dst, long long ldd, int wid,
                             int nwarps, int lane) {
  const int tm = (M + 3) >> 2, tn = (L.N + 31) >> 5;
  const float alpha = L.alpha_ptr ? *L.alpha_ptr : L.alpha;
  for (int t = wid; t < tm * tn; t += nwarps) {
    const int m0 = (t / tn) * 4, n = (t % tn) * 32 + lane;
    const float* wr = L.w + (long long)min(n, L.N - 1) * L.ldw;
    const float* xr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) xr[i] = x + (long long)min(m0 + i, M - 1) * ldx;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (VEC) {
#pragma unroll 4
      for (int k = 0; k < L.K; k += 4) {
        const float4 w = __ldg(reinterpret_cast<const float4*>(wr + k));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 a = __ldg(reinterpret_cast<const float4*>(xr[i] + k));
          acc[i] = fmaf(a.x, w.x, acc[i]);
          acc[i] = fmaf(a.y, w.y, acc[i]);
          acc[i] = fmaf(a.z, w.z, acc[i]);
          acc[i] = fmaf(a.w, w.w, acc[i]);
        }
      }
    } else {
      for (int k = 0; k < L.K; ++k) {
        const float w = __ldg(wr + k);
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] = fmaf(__ldg(xr[i] + k), w, acc[i]);
      }
    }
    if (n < L.N) {
      const float b = L.bias ? L.bias[(long long)n * L.bstride] : 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (m0 + i < M) dst[(long long)(m0 + i) * ldd + n] = act_apply_rt(L.act, acc[i] * alpha + b);
    }
  }
}

constexpr int kShortK = 256;

__global__ void __launch_bounds__(kSWarps * 32) small_mlp_kernel(SParams p) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gw = blockIdx.x * kSWarps + warp, nw = gridDim.x * kSWarps;
  float* dst1 = p.layers == 2 ? p.h : p.out;
  const long long ld1 = p.layers == 2 ? p.ldh : p.ldo;
  if (p.l1.K <= kShortK) {
    if (p.l1.vec) layer_rows32<true>(p.a, p.lda, p.M, p.l1, dst1, ld1, gw, nw, lane);
    else layer_rows32<false>(p.a, p.lda, p.M, p.l1, dst1, ld1, gw, nw, lane);
  } else if (p.l1.vec) {
    layer_tiles<true, 0, 0>(p.a, p.lda, p.M, p.l1, dst1, ld1, gw, nw, lane);
  } else {
    layer_tiles<false, 0, 0>(p.a, p.lda, p.M, p.l1, dst1, ld1, gw, nw, lane);
  }
  if (p.layers == 1) return;
  // The last CTA to arrive runs layer 2: its layer-1 rows are complete and,
  // after the fences, visible in L2 (read with ld.global.cg below).
  __shared__ int last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(p.counter, 1ull) == (unsigned long long)(gridDim.x - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (p.l2_smem) {
    // Layer 2 from shared memory: stage the layer-1 rows h [M][K2] and the
    // weight w2 [N2][K2] (eight loads in flight per thread), compute the
    // [M][N2] outputs with the warps' 4x4 blocks reading shared memory, then
    // the softmax reads them there too.
    extern __shared__ __align__(16) float sm[];
    const int K2 = p.l2.K, N2 = p.l2.N, M = p.M;
    float* hs = sm;                    // [M][K2]
    float* ws = hs + (size_t)M * K2;   // [N2][K2]
    float* zs = ws + (size_t)N2 * K2;  // [M][N2]
    constexpr int kBatch = 8;
    if (p.l2.vec) {
      const int q = K2 >> 2, nh = M * q, nall = nh + N2 * q;
      for (int i0 = threadIdx.x; i0 < nall; i0 += blockDim.x * kBatch) {
        float4 v[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int i = i0 + u * blockDim.x;
          if (i < nh) {
            const int m = i / q;
            v[u] = __ldcg(reinterpret_cast<const float4*>(p.h + (long long)m * p.ldh) + (i - m * q));
          } else if (i < nall) {
            const int n = (i - nh) / q;
            v[u] = __ldg(reinterpret_cast<const float4*>(p.l2.w + (long long)n * p.l2.ldw) + (i - nh - n * q));
          }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
          if (i0 + u * blockDim.x < nall) reinterpret_cast<float4*>(sm)[i0 + u * blockDim.x] = v[u];
      }
    } else {
      const int nh = M * K2, nall = nh + N2 * K2;
      for (int i0 = threadIdx.x; i0 < nall; i0 += blockDim.x * kBatch) {
        float v[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int i = i0 + u * blockDim.x;
          v[u] = 0.f;
          if (i < nh) {
            const int m = i / K2;
            v[u] = __ldcg(p.h + (long long)m * p.ldh + (i - m * K2));
          } else if (i < nall) {
            const int n = (i - nh) / K2;
            v[u] = __ldg(p.l2.w + (long long)n * p.l2.ldw + (i - nh - n * K2));
          }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
          if (i0 + u * blockDim.x < nall) sm[i0 + u * blockDim.x] = v[u];
      }
    }
    __syncthreads();
    SLayer l2s = p.l2;
    l2s.w = ws;
    l2s.ldw = K2;
    if (l2s.vec) layer_tiles<true, 2, 2>(hs, K2, M, l2s, zs, N2, warp, kSWarps, lane);
    else layer_tiles<false, 2, 2>(hs, K2, M, l2s, zs, N2, warp, kSWarps, lane);
    __syncthreads();
    for (int m = warp; m < M; m += kSWarps) {
      const float* zr = zs + m * N2;
      float* row = p.out + (long long)m * p.ldo;
      if (!p.softmax) {
        for (int n = lane; n < N2; n += 32) row[n] = zr[n];
        continue;
      }
      float mx = -__int_as_float(0x7f800000);
      for (int n = lane; n < N2; n += 32) mx = fmaxf(mx, zr[n]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      float sum = 0.f;
      for (int n = lane; n < N2; n += 32) sum += expf(zr[n] - mx);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      if (p.softmax == 1) {
        for (int n = lane; n < N2; n += 32) row[n] = expf(zr[n] - mx) / sum;
      } else {
        const float ls = logf(sum);
        for (int n = lane; n < N2; n += 32) row[n] = zr[n] - mx - ls;
      }
    }
    return;
  } else if (p.l2.vec) {
    layer_tiles<true, 1, 0>(p.h, p.ldh, p.M, p.l2, p.out, p.ldo, warp, kSWarps, lane);
  } else {
    layer_tiles<false, 1, 0>(p.h, p.ldh, p.M, p.l2, p.out, p.ldo, warp, kSWarps, lane);
  }
  if (!p.softmax) return;
  __syncthreads();  // this CTA's layer-2 stores are visible to all its threads
  const int N = p.l2.N;
  for (int m = warp; m < p.M; m += kSWarps) {
    float* row = p.out + (long long)m * p.ldo;
    float mx = -__int_as_float(0x7f800000);
    for (int n = lane; n < N; n += 32) mx = fmaxf(mx, row[n]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float s = 0.f;
    for (int n = lane; n < N; n += 32) s += expf(row[n] - mx);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (p.softmax == 1) {
      for (int n = lane; n < N; n += 32) row[n] = expf(row[n] - mx) / s;
    } else {
      const float ls = logf(s);
      for (int n = lane; n < N; n += 32) row[n] = row[n] - mx - ls;
    }
  }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// ---------------------------------------------------------------------------
// Two layers on clusters of kCluster CTAs.  The last-CTA scheme above leaves
// layer 2 and the softmax to one SM, whose loads of the layer-1 rows and
// serial work measured 20 of a 26 us launch at 64 x 784 -> 256 -> 10.  Here
// cluster g owns rows [gR, gR+R) and CTA c of it hidden units [cS, cS+S):
//   1. one 16-byte bulk copy per row brings the cluster's x rows and the CTA's
//      weight rows into shared memory (one memory round trip);
//   2. the warps' 4 x 4 blocks compute h = act1(alpha1 x W1^T + bias1) for
//      those rows and units from shared memory;
//   3. each CTA multiplies its slice of h by the matching columns of W2: a
//      partial [R][N2] sum, kept in its shared memory;
//   4. after a cluster barrier, CTA c sums the kCluster partials of rows
//      c, c+kCluster, ... (distributed shared memory, in rank order), applies
//      alpha2 / bias2 / act2 and the softmax, and writes the rows;
//   5. a last cluster barrier keeps every CTA's partials alive until read.
// No grid-wide dependency and no arrival counter; the summation order is
// fixed.
constexpr int kCluster = 8;
constexpr size_t kClusterSmemMax = 200 * 1024;
constexpr int kClusterMaxN2 = 256;

struct CParams {
  const float* a;
  long long lda;
  int M;
  SLayer l1, l2;
  float* out;
  long long ldo;
  int softmax;
  int R, S;  // rows per cluster, hidden units per CTA (a multiple of 4)
  int* err;
};

void cluster_shape(int64_t M, int64_t N1, int* R, int* S) {
  const int64_t G = std::min<int64_t>(16, (M + 3) / 4);  // at most 128 CTAs
  *R = (int)ceil_div(M, std::max<int64_t>(G, 1));
  *S = (int)(4 * ceil_div(N1, 4 * kCluster));
}
size_t cluster_smem(int R, int S, int64_t K, int64_t N2) {
  return ((size_t)(R + S) * (size_t)K + (size_t)R * S + (size_t)R * (size_t)N2) * sizeof(float) + 16;
}


__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kSWarps * 32) small_mlp_cluster_kernel(CParams p) {
  namespace cg = cooperative_groups;
  extern __shared__ __align__(16) unsigned char smc[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smc);
  const int K = p.l1.K, R = p.R, S = p.S, N2 = p.l2.N;
  float* xs = reinterpret_cast<float*>(smc + 16);  // [R][K]
  float* ws = xs + (size_t)R * K;                   // [S][K]
  float* hs = ws + (size_t)S * K;                   // [R][S]
  float* zp = hs + (size_t)R * S;                   // [R][N2] partial layer-2 sums
  cg::cluster_group cl = cg::this_cluster();
  const int c = (int)cl.block_rank();
  const int m0 = (blockIdx.x / kCluster) * R;
  const int rows = max(0, min(R, p.M - m0));
  const int j0 = c * S, cols = max(0, min(S, p.l1.N - j0));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(bar), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t bytes = (uint32_t)K * 4u;
    mbar_expect_tx(smem_u32(bar), bytes * (uint32_t)(rows + cols));
    for (int i = 0; i < rows; ++i)
      bulk_g2s(smem_u32(xs + (size_t)i * K), p.a + (long long)(m0 + i) * p.lda, bytes, smem_u32(bar));
    for (int i = 0; i < cols; ++i)
      bulk_g2s(smem_u32(ws + (size_t)i * K), p.l1.w + (long long)(j0 + i) * p.l1.ldw, bytes, smem_u32(bar));
  }
  // a copy that never lands is reported and waited for once more, bounded
  if (!mbar_wait(smem_u32(bar), 0u, p.err)) mbar_wait_own(smem_u32(bar), 0u, p.err);
  if (rows > 0 && cols > 0) {
    SLayer l1 = p.l1;
    l1.w = ws;
    l1.ldw = K;
    l1.N = cols;
    if (l1.bias) l1.bias += (long long)j0 * l1.bstride;
    layer_tiles<true, 2, 2>(xs, K, rows, l1, hs, S, warp, kSWarps, lane);
  }
  __syncthreads();
  // this CTA's share of layer 2: zp[m][n] = sum over its units j of h[m][j] * W2[n][j0 + j]
  for (int i = threadIdx.x; i < rows * N2; i += blockDim.x) {
    const int m = i / N2, n = i - m * N2;
    const float* hr = hs + (size_t)m * S;
    const float* wr = p.l2.w + (long long)n * p.l2.ldw + j0;
    float acc = 0.f;
    for (int j = 0; j < cols; j += 4) {
      if (j + 4 <= cols) {
        const float4 w4 = __ldg(reinterpret_cast<const float4*>(wr + j));
        const float4 h4 = *reinterpret_cast<const float4*>(hr + j);
        acc = fmaf(h4.x, w4.x, acc);
        acc = fmaf(h4.y, w4.y, acc);
        acc = fmaf(h4.z, w4.z, acc);
        acc = fmaf(h4.w, w4.w, acc);
      } else {
        for (int jj = j; jj < cols; ++jj) acc = fmaf(hr[jj], __ldg(wr + jj), acc);
      }
    }
    zp[i] = acc;
  }
  cl.sync();
  const float alpha2 = p.l2.alpha_ptr ? *p.l2.alpha_ptr : p.l2.alpha;
  for (int m = c + kCluster * warp; m < rows; m += kCluster * kSWarps) {
    float z[kClusterMaxN2 / 32];
#pragma unroll
    for (int k = 0; k < kClusterMaxN2 / 32; ++k) {
      const int n = lane + 32 * k;
      z[k] = -__int_as_float(0x7f800000);
      if (n < N2) {
        float sum = 0.f;
#pragma unroll
        for (int r = 0; r < kCluster; ++r) sum += cl.map_shared_rank(zp, r)[(size_t)m * N2 + n];
        float v = sum * alpha2;
        if (p.l2.bias) v += p.l2.bias[(long long)n * p.l2.bstride];
        z[k] = act_apply_rt(p.l2.act, v);
      }
    }
    float* row = p.out + (long long)(m0 + m) * p.ldo;
    if (!p.softmax) {
#pragma unroll
      for (int k = 0; k < kClusterMaxN2 / 32; ++k)
        if (lane + 32 * k < N2) row[lane + 32 * k] = z[k];
      continue;
    }
    float mx = -__int_as_float(0x7f800000);
#pragma unroll
    for (int k = 0; k < kClusterMaxN2 / 32; ++k)
      if (lane + 32 * k < N2) mx = fmaxf(mx, z[k]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < kClusterMaxN2 / 32; ++k)
      if (lane + 32 * k < N2) sum += expf(z[k] - mx);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (p.softmax == 1) {
#pragma unroll
      for (int k = 0; k < kClusterMaxN2 / 32; ++k)
        if (lane + 32 * k < N2) row[lane + 32 * k] = expf(z[k] - mx) / sum;
    } else {
      const float ls = logf(sum);
#pragma unroll
      for (int k = 0; k < kClusterMaxN2 / 32; ++k)
        if (lane + 32 * k < N2) row[lane + 32 * k] = z[k] - mx - ls;
    }
  }
  cl.sync();  // the partials stay in shared memory until every CTA has read them
}

}  // namespace

bool small_mlp_cluster_fits(int64_t M, int64_t N1, int64_t K1, int64_t N2) {
  if (M < 1 || M > kSmallMaxRows || N1 < 1 || K1 < 4 || K1 % 4 != 0 || N2 < 1 || N2 > kClusterMaxN2) return false;
  int R, S;
  cluster_shape(M, N1, &R, &S);
  return cluster_smem(R, S, K1, N2) <= kClusterSmemMax;
}

void launch_small_mlp(const SmallMlpLaunch& L, cudaStream_t stream) {
  PFB_CHECK_ARG(L.M > 0 && L.M <= kSmallMaxRows, "small GEMM: 1..256 rows");
  PFB_CHECK_ARG(L.layers == 1 || L.layers == 2, "small GEMM: one or two layers");
  PFB_CHECK_ARG(L.a && L.w1 && L.out && L.N1 > 0 && L.K1 > 0 && L.lda >= L.K1 && L.ldw1 >= L.K1,
                "small GEMM: bad layer-1 operands");
  PFB_CHECK_ARG(L.K1 < (1 << 24) && L.N1 < (1 << 20), "small GEMM: layer too large");
  SParams p{};
  p.a = L.a;
  p.lda = L.lda;
  p.M = (int)L.M;
  p.layers = L.layers;
  p.out = L.out;
  p.ldo = L.ldo;
  p.softmax = L.softmax;
  auto layer = [](SLayer& s, const float* w, int64_t ldw, const float* bias, int64_t bstride, float alpha,
                  const float* alpha_ptr, int64_t N, int64_t K, int act, const float* x, int64_t ldx) {
    s.w = w;
    s.ldw = ldw;
    s.bias = bias;
    s.bstride = bstride;
    s.alpha = alpha;
    s.alpha_ptr = alpha_ptr;
    s.N = (int)N;
    s.K = (int)K;
    s.act = act;
    s.vec = K % 4 == 0 && ldw % 4 == 0 && ldx % 4 == 0 && aligned16(w) && aligned16(x);
  };
  layer(p.l1, L.w1, L.ldw1, L.bias1, L.bstride1, L.alpha1, L.alpha1_ptr, L.N1, L.K1, L.act1, L.a, L.lda);
  if (L.layers == 2) {
    PFB_CHECK_ARG(L.w2 && (L.cluster || (L.h && L.counter && L.ldh >= L.N1)) && L.N2 > 0 && L.ldw2 >= L.N1 &&
                      L.N2 < (1 << 20),
                  "small GEMM: bad layer-2 operands");
    layer(p.l2, L.w2, L.ldw2, L.bias2, L.bstride2, L.alpha2, L.alpha2_ptr, L.N2, L.N1, L.act2, L.h, L.ldh);
    p.h = L.h;
    p.ldh = L.ldh;
    p.counter = L.counter;
    PFB_CHECK_ARG(L.ldo >= L.N2, "small GEMM: output pitch below the row length");
  } else {
    PFB_CHECK_ARG(L.softmax == 0, "small GEMM: a fused softmax needs two layers");
    PFB_CHECK_ARG(L.ldo >= L.N1, "small GEMM: output pitch below the row length");
  }
  if (L.cluster) {
    PFB_CHECK_ARG(L.layers == 2 && small_mlp_cluster_fits(L.M, L.N1, L.K1, L.N2) && L.err && p.l1.vec &&
                      L.ldw2 % 4 == 0 && aligned16(L.w2) && L.softmax >= 0 && L.softmax <= 2,
                  "small MLP on clusters: unaligned rows or sizes past the shared-memory staging");
    CParams c;
    c.a = L.a;
    c.lda = L.lda;
    c.M = (int)L.M;
    c.l1 = p.l1;
    c.l2 = p.l2;
    c.out = L.out;
    c.ldo = L.ldo;
    c.softmax = L.softmax;
    c.err = L.err;
    cluster_shape(L.M, L.N1, &c.R, &c.S);
    const size_t smem = cluster_smem(c.R, c.S, L.K1, L.N2);
    const int dev = current_device();
    static std::once_flag attr_once[64];
    std::call_once(attr_once[dev], [] {
      PFB_CUDA(cudaFuncSetAttribute(small_mlp_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kClusterSmemMax));
    });
    const unsigned clusters = (unsigned)ceil_div(L.M, (int64_t)c.R);
    small_mlp_cluster_kernel<<<clusters * kCluster, kSWarps * 32, smem, stream>>>(c);
    PFB_CUDA(cudaGetLastError());
    return;
  }
  size_t smem = 0;
  if (L.layers == 2) {
    const size_t need = ((size_t)(L.M + L.N2) * (size_t)L.N1 + (size_t)L.M * (size_t)L.N2) * sizeof(float);
    if (need <= kSmallSmemMax) {
      p.l2_smem = 1;
      smem = need;
    }
  }
  const int dev = current_device();
  static std::once_flag attr_once[64];
  std::call_once(attr_once[dev], [] {
    PFB_CUDA(cudaFuncSetAttribute(small_mlp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmallSmemMax));
  });
  const int64_t tiles = ((L.M + 3) / 4) * (L.K1 <= kShortK ? (L.N1 + 31) / 32 : (L.N1 + 3) / 4);
  const int64_t sms = device_sm_count(dev);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((tiles + kSWarps - 1) / kSWarps, 4 * sms));
  small_mlp_kernel<<<grid, kSWarps * 32, smem, stream>>>(p);
  PFB_CUDA(cudaGetLastError());
}

}  // namespace pfb
