// Memory-bound kernels around the tensor-core GEMM: operand preparation
// (fp32 -> tf32 hi/lo split or bf16, K-major, zero-padded K), im2col for
// Conv2d as implicit GEMM, pooling, and BatchNorm(eval) folding.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "../common.hpp"
#include "kernels.hpp"
#include "split.cuh"

namespace pfb {

namespace {

int num_sms() { return device_sm_count(current_device()); }

unsigned grid_for(int64_t work, int block) {
  int64_t g = ceil_div(std::max<int64_t>(work, 1), block);
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(g, (int64_t)num_sms() * 32));
}

struct View6 {
  int rank;
  long long shape[6];
  long long stride[6];
};

__device__ __forceinline__ long long row_offset(const View6& v, long long row) {
  // rows enumerate dims [0, rank-1) row-major
  long long off = 0;
  for (int d = v.rank - 2; d >= 0; --d) {
    long long sz = v.shape[d];
    off += (row % sz) * v.stride[d];
    row /= sz;
  }
  return off;
}

// Generic path: one output element per thread (k fastest, coalesced writes).
template <int PREC>
__global__ void prepare_generic(const float* __restrict__ src, View6 v, long long rows, long long kpad,
                                void* __restrict__ hi, float* __restrict__ lo) {
  const long long K = v.shape[v.rank - 1];
  const long long sk = v.stride[v.rank - 1];
  const long long total = rows * kpad;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / kpad, k = i % kpad;
    float x = 0.f;
    if (k < K) x = src[row_offset(v, r) + k * sk];
    if constexpr (PREC == PFC_PRECISION_BF16) {
      ((__nv_bfloat16*)hi)[i] = __float2bfloat16_rn(x);
    } else {
      float h, l;
      split_tf32(x, h, l);
      ((float*)hi)[i] = h;
      lo[i] = l;
    }
  }
}

// Vector path: K contiguous (stride 1), K % 4 == 0, 16-byte aligned rows.
template <int PREC>
__global__ void prepare_vec4(const float* __restrict__ src, View6 v, long long rows, long long kpad,
                             void* __restrict__ hi, float* __restrict__ lo) {
  const long long K = v.shape[v.rank - 1];
  const long long kq = kpad / 4;
  const long long total = rows * kq;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / kq, k = (i % kq) * 4;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (k < K) x = *(const float4*)(src + row_offset(v, r) + k);
    const long long o = r * kpad + k;
    if constexpr (PREC == PFC_PRECISION_BF16) {
      __nv_bfloat162 a = __floats2bfloat162_rn(x.x, x.y), b = __floats2bfloat162_rn(x.z, x.w);
      uint2 pk;
      pk.x = *(uint32_t*)&a;
      pk.y = *(uint32_t*)&b;
      *(uint2*)((__nv_bfloat16*)hi + o) = pk;
    } else {
      float4 h, l;
      split_tf32(x.x, h.x, l.x);
      split_tf32(x.y, h.y, l.y);
      split_tf32(x.z, h.z, l.z);
      split_tf32(x.w, h.w, l.w);
      *(float4*)((float*)hi + o) = h;
      *(float4*)(lo + o) = l;
    }
  }
}

// Dense row-major source with kpad == K: the operand is the source split
// element for element, one float4 per thread step and no index arithmetic
// (the general path's 64-bit row/column divisions made it instruction-bound).
template <int PREC>
__global__ void prepare_flat4(const float4* __restrict__ src, long long n4, void* __restrict__ hi,
                              float* __restrict__ lo) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const float4 x = src[i];
    if constexpr (PREC == PFC_PRECISION_BF16) {
      __nv_bfloat162 a = __floats2bfloat162_rn(x.x, x.y), b = __floats2bfloat162_rn(x.z, x.w);
      uint2 pk;
      pk.x = *(uint32_t*)&a;
      pk.y = *(uint32_t*)&b;
      reinterpret_cast<uint2*>(hi)[i] = pk;
    } else {
      float4 h, l;
      split_tf32(x.x, h.x, l.x);
      split_tf32(x.y, h.y, l.y);
      split_tf32(x.z, h.z, l.z);
      split_tf32(x.w, h.w, l.w);
      reinterpret_cast<float4*>(hi)[i] = h;
      reinterpret_cast<float4*>(lo)[i] = l;
    }
  }
}

// Transposed source: the last row dim is contiguous (stride 1) and K is
// strided.  32x32 tiles through shared memory keep both sides coalesced.
template <int PREC>
__global__ void prepare_transpose(const float* __restrict__ src, View6 v, long long rows, long long kpad,
                                  void* __restrict__ hi, float* __restrict__ lo) {
  __shared__ float tile[32][33];
  const long long K = v.shape[v.rank - 1];
  const long long sk = v.stride[v.rank - 1];
  const long long R = v.shape[v.rank - 2];  // innermost row dim (contiguous)
  const long long outer = rows / R;
  const long long tiles_r = (R + 31) / 32, tiles_k = (kpad + 31) / 32;
  const long long ntiles = outer * tiles_r * tiles_k;
  for (long long t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const long long tk = t % tiles_k, tr = (t / tiles_k) % tiles_r, ob = t / (tiles_k * tiles_r);
    const long long base = row_offset(v, ob * R);  // offset of (ob, r=0)
    // load: threadIdx.x walks r (contiguous in memory)
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
      const long long k = tk * 32 + j, r = tr * 32 + threadIdx.x;
      float x = 0.f;
      if (k < K && r < R) x = src[base + r * v.stride[v.rank - 2] + k * sk];
      tile[j][threadIdx.x] = x;
    }
    __syncthreads();
    // store: threadIdx.x walks k (contiguous in the output)
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
      const long long r = tr * 32 + j, k = tk * 32 + threadIdx.x;
      if (r < R && k < kpad) {
        const float x = tile[threadIdx.x][j];
        const long long o = (ob * R + r) * kpad + k;
        if constexpr (PREC == PFC_PRECISION_BF16) {
          ((__nv_bfloat16*)hi)[o] = __float2bfloat16_rn(x);
        } else {
          float h, l;
          split_tf32(x, h, l);
          ((float*)hi)[o] = h;
          lo[o] = l;
        }
      }
    }
    __syncthreads();
  }
}

template <int PREC>
__global__ void im2col_kernel(const float* __restrict__ x, Im2colLaunch L, void* __restrict__ hi, float* __restrict__ lo) {
  const long long K = L.c * L.kh * L.kw;
  const long long M = L.n * L.oh * L.ow;
  const long long total = M * L.kpad;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / L.kpad, k = i % L.kpad;
    float v = 0.f;
    if (k < K) {
      const long long ow = m % L.ow, oh = (m / L.ow) % L.oh, n = m / (L.ow * L.oh);
      const long long kw = k % L.kw, kh = (k / L.kw) % L.kh, c = k / (L.kw * L.kh);
      const long long ih = oh * L.stride_h - L.pad_h + kh * L.dil_h;
      const long long iw = ow * L.stride_w - L.pad_w + kw * L.dil_w;
      if (ih >= 0 && ih < L.h && iw >= 0 && iw < L.w) v = x[n * L.sn + c * L.sc + ih * L.sh + iw * L.sw];
    }
    if constexpr (PREC == PFC_PRECISION_BF16) {
      ((__nv_bfloat16*)hi)[i] = __float2bfloat16_rn(v);
    } else {
      float h, l;
      split_tf32(v, h, l);
      ((float*)hi)[i] = h;
      lo[i] = l;
    }
  }
}

// Pooling (pooling.cpp:38-63,97-122,150-168): one output element per thread,
// enumerated channel-fastest when the output is channels-last.
// grid.y walks output rows (n, oh); threads walk (ow, c) of a row with 32-bit
// index math, channel fastest for a channels-last output (coalesced reads of
// a channels-last input and coalesced writes), column fastest otherwise.
__global__ void pool_kernel(PoolLaunch L) {
  const bool cl = L.osc == 1;  // channels-last output
  const int C = (int)L.c, OW = (int)L.ow;
  const int inner = C * OW;
  for (long long row = blockIdx.y; row < L.n * L.oh; row += gridDim.y) {
   const long long n = row / L.oh, oh = row - n * L.oh;
   for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < inner; i += gridDim.x * blockDim.x) {
    long long c, ow;
    if (cl) {
      c = i % C; ow = i / C;
    } else {
      ow = i % OW; c = i / OW;
    }
    const float* xb = L.x + n * L.sn + c * L.sc;
    float out;
    if (L.mode == 2) {
      // adaptive average: window [floor(i*H/OH), ceil((i+1)*H/OH))
      const long long h0 = (oh * L.h) / L.oh, h1 = ((oh + 1) * L.h + L.oh - 1) / L.oh;
      const long long w0 = (ow * L.w) / L.ow, w1 = ((ow + 1) * L.w + L.ow - 1) / L.ow;
      float s = 0.f;
      for (long long h = h0; h < h1; ++h)
        for (long long w = w0; w < w1; ++w) s += xb[h * L.sh + w * L.sw];
      out = s / (float)((h1 - h0) * (w1 - w0));
    } else {
      const long long hs = oh * L.stride_h - L.pad_h, ws = ow * L.stride_w - L.pad_w;
      if (L.mode == 0) {
        float m = -__int_as_float(0x7f800000);
        for (long long kh = 0; kh < L.kh; ++kh) {
          const long long h = hs + kh;
          if (h < 0 || h >= L.h) continue;
          for (long long kw = 0; kw < L.kw; ++kw) {
            const long long w = ws + kw;
            if (w < 0 || w >= L.w) continue;
            const float v = xb[h * L.sh + w * L.sw];
            if (v > m || isnan(v)) m = v;
          }
        }
        out = m;
      } else {
        float s = 0.f;
        for (long long kh = 0; kh < L.kh; ++kh) {
          const long long h = hs + kh;
          if (h < 0 || h >= L.h) continue;
          for (long long kw = 0; kw < L.kw; ++kw) {
            const long long w = ws + kw;
            if (w < 0 || w >= L.w) continue;
            s += xb[h * L.sh + w * L.sw];
          }
        }
        out = s / (float)(L.kh * L.kw);  // count includes padding
      }
    }
    const long long yo = n * L.osn + c * L.osc + oh * L.osh + ow * L.osw;
    if (L.y) L.y[yo] = out;
    if (L.out_hi) {
      if (L.precision == PFC_PRECISION_BF16) {
        ((__nv_bfloat16*)L.out_hi)[yo] = __float2bfloat16_rn(out);
      } else {
        float hv, lv;
        split_tf32(out, hv, lv);
        ((float*)L.out_hi)[yo] = hv;
        L.out_lo[yo] = lv;
      }
    }
   }
  }
}

// Channels-last copy of a Conv2d input: one thread per pixel and group of 4
// channels (float4 stores, coalesced; the 4 reads are coalesced across
// threads for channels-last and channel-planar inputs alike).  IDX is int
// when every index fits in 32 bits.
template <int PREC, typename IDX>
__global__ void conv_input_kernel(ConvInputLaunch L) {
  // output extent: the padded image when hp > 0 (zeros outside the input).
  // One thread per output pixel, walking its Cp/4 channel groups: lanes take
  // neighbouring pixels, so an NCHW source is read along its channel planes
  // (coalesced) and each pixel's index arithmetic is paid once.
  const IDX C = (IDX)L.c, G = (IDX)(L.cp / 4), H = (IDX)L.h, W = (IDX)L.w;
  const IDX OHp = L.hp > 0 ? (IDX)L.hp : H, OWp = L.hp > 0 ? (IDX)L.wp : W;
  const IDX PH = L.hp > 0 ? (IDX)L.ph : 0, PW = L.hp > 0 ? (IDX)L.pw : 0;
  const IDX total = (IDX)L.n * OHp * OWp;
  const IDX half = OWp / 2;
  for (IDX pix = (IDX)blockIdx.x * blockDim.x + threadIdx.x; pix < total; pix += (IDX)gridDim.x * blockDim.x) {
    const IDX wq = pix % OWp;
    const IDX hn = pix / OWp;
    // destination pixel: de-interleaved rows keep even columns, then odd ones
    const IDX dpix = L.deint ? hn * OWp + (wq & 1) * half + (wq >> 1) : pix;
    const IDX hq = hn % OHp;
    const IDX n = hn / OHp;
    const IDX h = hq - PH, w = wq - PW;
    const bool inside = h >= 0 && h < H && w >= 0 && w < W;
    const float* src = L.x + (long long)n * L.sn + (long long)h * L.sh + (long long)w * L.sw;
    auto group = [&](IDX g, float (&x)[4]) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const IDX c = 4 * g + j;
        x[j] = (inside && c < C) ? src[(long long)c * L.sc] : 0.f;
      }
    };
    if constexpr (PREC == PFC_PRECISION_BF16) {
      // pairs of groups as one 16-byte store (Cp is a multiple of 8 here)
      for (IDX g = 0; g < G; g += 2) {
        float x[4], y[4];
        group(g, x);
        group(g + 1, y);
        const __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]), b = __floats2bfloat162_rn(x[2], x[3]);
        const __nv_bfloat162 c = __floats2bfloat162_rn(y[0], y[1]), d = __floats2bfloat162_rn(y[2], y[3]);
        uint4 pk;
        pk.x = *(const uint32_t*)&a;
        pk.y = *(const uint32_t*)&b;
        pk.z = *(const uint32_t*)&c;
        pk.w = *(const uint32_t*)&d;
        *(uint4*)((__nv_bfloat16*)L.hi + 4 * (dpix * G + g)) = pk;
      }
    } else {
      for (IDX g = 0; g < G; ++g) {
        float x[4];
        group(g, x);
        float4 hv, lv;
        split_tf32(x[0], hv.x, lv.x);
        split_tf32(x[1], hv.y, lv.y);
        split_tf32(x[2], hv.z, lv.z);
        split_tf32(x[3], hv.w, lv.w);
        *(float4*)((float*)L.hi + 4 * (dpix * G + g)) = hv;
        *(float4*)(L.lo + 4 * (dpix * G + g)) = lv;
      }
    }
  }
}

// Conv2d weight [O,C,KH,KW] -> [O][kpad], k = (kh*KW + kw)*Cp + c.
template <int PREC>
__global__ void conv_weight_kernel(ConvWeightLaunch L) {
  const long long total = L.o * L.kpad;
  const long long kwp = L.kwp > 0 ? L.kwp : L.kw;  // taps per filter row in the layout
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long o = i / L.kpad, k = i % L.kpad;
    const long long slot = k / L.cp, c = k % L.cp;
    const long long kh = slot / kwp, kw = slot % kwp;
    float x = 0.f;
    if (kh < L.kh && kw < L.kw && c < L.c) x = L.w[o * L.so + c * L.sc + kh * L.skh + kw * L.skw];
    if constexpr (PREC == PFC_PRECISION_BF16) {
      ((__nv_bfloat16*)L.hi)[i] = __float2bfloat16_rn(x);
    } else {
      float hv, lv;
      split_tf32(x, hv, lv);
      ((float*)L.hi)[i] = hv;
      L.lo[i] = lv;
    }
  }
}

// Max / average pool on channels-last data (input and output channel
// stride 1, C % 4 == 0): grid.y walks output rows (n, oh), threads take 4
// channels of one output column each (float4 loads and stores, 32-bit index
// math inside an image, window clipped once).  Same NaN rule and window order
// as pool_kernel.
__global__ void pool_cl_kernel(PoolLaunch L) {
  const int C4 = (int)(L.c / 4), OW = (int)L.ow, OH = (int)L.oh;
  const int H = (int)L.h, W = (int)L.w, sh = (int)L.sh, sw = (int)L.sw;
  const int inner = C4 * OW;
  const int rows = (int)(L.n * L.oh);
  for (int row = blockIdx.y; row < rows; row += gridDim.y) {
    const int n = row / OH, oh = row - n * OH;
    const float* xb = L.x + (long long)n * L.sn;
    const int hs = oh * (int)L.stride_h - (int)L.pad_h;
    const int h0 = max(hs, 0), h1 = min(hs + (int)L.kh, H);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < inner; i += gridDim.x * blockDim.x) {
      const int c = (i % C4) * 4, ow = i / C4;
      const int ws = ow * (int)L.stride_w - (int)L.pad_w;
      const int w0 = max(ws, 0), w1 = min(ws + (int)L.kw, W);
      float r[4];
      if (L.mode == 0 && h1 - h0 == 3 && w1 - w0 == 3) {
        // a whole 3x3 window: all nine loads in flight, then the same
        // NaN-aware max in the same (h, w) order
        const float* base = xb + h0 * sh + w0 * sw + c;
        float4 v4[9];
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
          for (int e = 0; e < 3; ++e) v4[a * 3 + e] = *reinterpret_cast<const float4*>(base + a * sh + e * sw);
#pragma unroll
        for (int j = 0; j < 4; ++j) r[j] = -__int_as_float(0x7f800000);
#pragma unroll
        for (int k = 0; k < 9; ++k) {
          const float v[4] = {v4[k].x, v4[k].y, v4[k].z, v4[k].w};
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (v[j] > r[j] || isnan(v[j])) r[j] = v[j];
        }
      } else if (L.mode == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) r[j] = -__int_as_float(0x7f800000);
        for (int h = h0; h < h1; ++h)
          for (int w = w0; w < w1; ++w) {
            const float4 v4 = *reinterpret_cast<const float4*>(xb + h * sh + w * sw + c);
            const float v[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j)
              if (v[j] > r[j] || isnan(v[j])) r[j] = v[j];
          }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) r[j] = 0.f;
        for (int h = h0; h < h1; ++h)
          for (int w = w0; w < w1; ++w) {
            const float4 v4 = *reinterpret_cast<const float4*>(xb + h * sh + w * sw + c);
            r[0] += v4.x; r[1] += v4.y; r[2] += v4.z; r[3] += v4.w;
          }
        const float cnt = (float)(L.kh * L.kw);  // count includes padding
#pragma unroll
        for (int j = 0; j < 4; ++j) r[j] = r[j] / cnt;
      }
      const long long yo = (long long)n * L.osn + (long long)oh * L.osh + (long long)ow * L.osw + c;
      if (L.y) *reinterpret_cast<float4*>(L.y + yo) = make_float4(r[0], r[1], r[2], r[3]);
      if (L.out_hi) {
        if (L.precision == PFC_PRECISION_BF16) {
#pragma unroll
          for (int j = 0; j < 4; ++j) ((__nv_bfloat16*)L.out_hi)[yo + j] = __float2bfloat16_rn(r[j]);
        } else {
          float4 hv, lv;
          split_tf32(r[0], hv.x, lv.x);
          split_tf32(r[1], hv.y, lv.y);
          split_tf32(r[2], hv.z, lv.z);
          split_tf32(r[3], hv.w, lv.w);
          *reinterpret_cast<float4*>((float*)L.out_hi + yo) = hv;
          *reinterpret_cast<float4*>(L.out_lo + yo) = lv;
        }
      }
    }
  }
}

// Adaptive average pool to 1x1 over a channels-last input: one CTA per
// (image, 32-channel group); 32 warps take every 32nd pixel, lanes are
// channels (coalesced 128-byte reads); the 32 partial sums meet in shared
// memory.
__global__ void __launch_bounds__(1024) global_avg_cl_kernel(PoolLaunch L) {
  __shared__ float part[32][33];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const long long n = blockIdx.y, c = (long long)blockIdx.x * 32 + lane;
  const long long P = L.h * L.w;
  float s = 0.f;
  if (c < L.c) {
    const float* xb = L.x + n * L.sn + c;
    for (long long p = wp; p < P; p += 32) {
      const long long h = p / L.w, w = p - h * L.w;
      s += xb[h * L.sh + w * L.sw];
    }
  }
  part[wp][lane] = s;
  __syncthreads();
  if (wp == 0 && c < L.c) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 32; ++k) t += part[k][lane];
    const float out = t / (float)P;
    const long long yo = n * L.osn + c * L.osc;
    if (L.y) L.y[yo] = out;
    if (L.out_hi) {
      if (L.precision == PFC_PRECISION_BF16) {
        ((__nv_bfloat16*)L.out_hi)[yo] = __float2bfloat16_rn(out);
      } else {
        float hv, lv;
        split_tf32(out, hv, lv);
        ((float*)L.out_hi)[yo] = hv;
        L.out_lo[yo] = lv;
      }
    }
  }
}

// Adaptive average pool to 1x1 over a dense channels-last image ([H*W][C],
// C % 4 == 0, C <= 1024): one 256-thread CTA per image.  Thread t takes the
// float4 of channels 4*(t % C4) of pixels t / C4, t / C4 + R, ... (R = 256 /
// C4 pixels per pass, four loads in flight), then the R partial sums of each
// channel combine through shared memory in a fixed order.
__global__ void __launch_bounds__(256) global_avg_cl4_kernel(PoolLaunch L) {
  __shared__ float4 part[256];
  const int C4 = (int)(L.c / 4), R = 256 / C4;
  const int t = threadIdx.x, j = t % C4, r = t / C4;
  const long long n = blockIdx.x;
  const int P = (int)(L.h * L.w);
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (r < R) {
    const float4* xb = reinterpret_cast<const float4*>(L.x + n * L.sn) + j;
    int p = r;
    for (; p + 3 * R < P; p += 4 * R) {
      const float4 a = xb[(long long)p * C4], b = xb[(long long)(p + R) * C4];
      const float4 c = xb[(long long)(p + 2 * R) * C4], d = xb[(long long)(p + 3 * R) * C4];
      s.x += a.x + b.x + c.x + d.x;
      s.y += a.y + b.y + c.y + d.y;
      s.z += a.z + b.z + c.z + d.z;
      s.w += a.w + b.w + c.w + d.w;
    }
    for (; p < P; p += R) {
      const float4 a = xb[(long long)p * C4];
      s.x += a.x; s.y += a.y; s.z += a.z; s.w += a.w;
    }
  }
  part[t] = s;
  __syncthreads();
  if (r == 0) {
    for (int k = 1; k < R; ++k) {
      const float4 o = part[k * C4 + j];
      s.x += o.x; s.y += o.y; s.z += o.z; s.w += o.w;
    }
    const float inv = 1.f / (float)P;
    const float out[4] = {s.x * inv, s.y * inv, s.z * inv, s.w * inv};
    for (int q = 0; q < 4; ++q) {
      const long long c = 4 * j + q;
      const long long yo = n * L.osn + c * L.osc;
      if (L.y) L.y[yo] = out[q];
      if (L.out_hi) {
        if (L.precision == PFC_PRECISION_BF16) {
          ((__nv_bfloat16*)L.out_hi)[yo] = __float2bfloat16_rn(out[q]);
        } else {
          float hv, lv;
          split_tf32(out[q], hv, lv);
          ((float*)L.out_hi)[yo] = hv;
          L.out_lo[yo] = lv;
        }
      }
    }
  }
}

// Global average pool finished from a convolution's per-tile column sums
// (PoolLaunch mode 3): one 512-thread CTA per image.  For each block of 64
// channels, eight thread groups add an eighth of the image's slots each
// (eight loads in flight per thread, coalesced across channels), and the
// eight parts are added in part order: a fixed summation order.
__global__ void __launch_bounds__(512) gap_finish_kernel(PoolLaunch L) {
  __shared__ float part[8][64];
  const int t = threadIdx.x, cl = t & 63, g = t >> 6;
  const long long n = blockIdx.x;
  const long long r0 = L.h * g / 8, r1 = L.h * (g + 1) / 8;
  for (long long c0 = 0; c0 < L.c; c0 += 64) {
    const long long c = c0 + cl;
    float s = 0.f;
    if (c < L.c) {
      const float* xb = L.x + n * L.sn + c * L.sc;
      float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      long long r = r0;
      for (; r + 7 < r1; r += 8) {
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] += xb[(r + k) * L.sh];
      }
      for (; r < r1; ++r) a[0] += xb[r * L.sh];
      s = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
    }
    part[g][cl] = s;
    __syncthreads();
    if (g == 0 && c < L.c) {
      float tot = part[0][cl];
#pragma unroll
      for (int k = 1; k < 8; ++k) tot += part[k][cl];
      const float out = tot / (float)L.count;
      const long long yo = n * L.osn + c * L.osc;
      if (L.y) L.y[yo] = out;
      if (L.out_hi) {
        if (L.precision == PFC_PRECISION_BF16) {
          ((__nv_bfloat16*)L.out_hi)[yo] = __float2bfloat16_rn(out);
        } else {
          float hv, lv;
          split_tf32(out, hv, lv);
          ((float*)L.out_hi)[yo] = hv;
          L.out_lo[yo] = lv;
        }
      }
    }
    __syncthreads();
  }
}

__global__ void bn_fold_kernel(BnFoldLaunch L) {
  for (long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x; c < L.channels; c += (long long)gridDim.x * blockDim.x) {
    const float g = L.gamma ? L.gamma[c * L.gs] : L.gamma_c;
    const float b = L.beta ? L.beta[c * L.bs] : L.beta_c;
    const float m = L.mean ? L.mean[c * L.ms] : L.mean_c;
    const float v = L.var ? L.var[c * L.vs] : L.var_c;
    const float cb = L.bias ? L.bias[c * L.cs] : L.bias_c;
    const float s = g / sqrtf(v + L.eps);
    L.scale[c] = s;
    L.shift[c] = (cb - m) * s + b;
  }
}

}  // namespace

void launch_prepare(const PrepLaunch& L, cudaStream_t stream) {
  PFB_CHECK_ARG(L.rank >= 1 && L.rank <= 6, "prepare: rank must be 1..6");
  View6 v;
  v.rank = L.rank;
  long long rows = 1;
  for (int d = 0; d < L.rank; ++d) {
    v.shape[d] = L.shape[d];
    v.stride[d] = L.stride[d];
    if (d + 1 < L.rank) rows *= L.shape[d];
  }
  if (L.rank == 1) {  // a single row
    v.rank = 2;
    v.shape[1] = v.shape[0];
    v.stride[1] = v.stride[0];
    v.shape[0] = 1;
    v.stride[0] = 0;
  }
  const long long K = v.shape[v.rank - 1];
  const long long sk = v.stride[v.rank - 1];
  if (rows * L.kpad == 0) return;
  const bool bf = L.precision == PFC_PRECISION_BF16;
  bool vec = sk == 1 && K % 4 == 0 && ((uintptr_t)L.src & 15) == 0;
  for (int d = 0; d + 1 < v.rank && vec; ++d) vec = (v.stride[d] % 4) == 0 || v.shape[d] == 1;
  const bool trans = !vec && sk != 1 && v.stride[v.rank - 2] == 1 && v.shape[v.rank - 2] > 1;
  bool dense = vec && L.kpad == K;
  {
    long long expect = K;
    for (int d = v.rank - 2; d >= 0 && dense; --d) {
      if (v.shape[d] != 1 && v.stride[d] != expect) dense = false;
      expect *= v.shape[d];
    }
  }
  if (dense) {
    const long long n4 = rows * K / 4;
    unsigned g = grid_for(n4, 256);
    if (bf) prepare_flat4<PFC_PRECISION_BF16><<<g, 256, 0, stream>>>((const float4*)L.src, n4, L.hi, L.lo);
    else prepare_flat4<PFC_PRECISION_TF32X3><<<g, 256, 0, stream>>>((const float4*)L.src, n4, L.hi, L.lo);
  } else if (vec) {
    unsigned g = grid_for(rows * (L.kpad / 4), 256);
    if (bf) prepare_vec4<PFC_PRECISION_BF16><<<g, 256, 0, stream>>>(L.src, v, rows, L.kpad, L.hi, L.lo);
    else prepare_vec4<PFC_PRECISION_TF32X3><<<g, 256, 0, stream>>>(L.src, v, rows, L.kpad, L.hi, L.lo);
  } else if (trans) {
    const long long R = v.shape[v.rank - 2];
    long long ntiles = (rows / R) * ceil_div(R, 32) * ceil_div(L.kpad, 32);
    unsigned g = (unsigned)std::max<long long>(1, std::min<long long>(ntiles, (long long)num_sms() * 16));
    dim3 blk(32, 8);
    if (bf) prepare_transpose<PFC_PRECISION_BF16><<<g, blk, 0, stream>>>(L.src, v, rows, L.kpad, L.hi, L.lo);
    else prepare_transpose<PFC_PRECISION_TF32X3><<<g, blk, 0, stream>>>(L.src, v, rows, L.kpad, L.hi, L.lo);
  } else {
    unsigned g = grid_for(rows * L.kpad, 256);
    if (bf) prepare_generic<PFC_PRECISION_BF16><<<g, 256, 0, stream>>>(L.src, v, rows, L.kpad, L.hi, L.lo);
    else prepare_generic<PFC_PRECISION_TF32X3><<<g, 256, 0, stream>>>(L.src, v, rows, L.kpad, L.hi, L.lo);
  }
  PFB_CUDA(cudaGetLastError());
}

void launch_im2col(const Im2colLaunch& L, cudaStream_t stream) {
  const long long total = L.n * L.oh * L.ow * L.kpad;
  if (total == 0) return;
  unsigned g = grid_for(total, 256);
  if (L.precision == PFC_PRECISION_BF16) im2col_kernel<PFC_PRECISION_BF16><<<g, 256, 0, stream>>>(L.x, L, L.hi, L.lo);
  else im2col_kernel<PFC_PRECISION_TF32X3><<<g, 256, 0, stream>>>(L.x, L, L.hi, L.lo);
  PFB_CUDA(cudaGetLastError());
}

void launch_pool(const PoolLaunch& L, cudaStream_t stream) {
  const long long total = L.n * L.c * L.oh * L.ow;
  if (total == 0) return;
  PFB_CHECK_ARG(L.c * L.ow < (1ll << 31), "pool: channels x output width too large");
  PFB_CHECK_ARG(L.y || L.out_hi, "pool: no output");
  PFB_CHECK_ARG(!L.out_hi || (L.osc == 1 && L.osw == L.c && L.osh == L.ow * L.c && L.osn == L.oh * L.ow * L.c &&
                              (L.precision == PFC_PRECISION_BF16 || L.out_lo)),
                "pool: operand output needs a dense channels-last layout");
  if (L.mode == 3) {
    PFB_CHECK_ARG(L.oh == 1 && L.ow == 1 && L.w == 1 && L.count > 0 && L.n < (1ll << 31),
                  "pool: a finished global average needs 1x1 outputs and a pixel count");
    gap_finish_kernel<<<(unsigned)L.n, 512, 0, stream>>>(L);
    PFB_CUDA(cudaGetLastError());
    return;
  }
  if (L.mode == 2 && L.oh == 1 && L.ow == 1 && L.sc == 1 && L.sw == L.c && L.sh == L.w * L.c && L.c % 4 == 0 &&
      L.c <= 1024 && L.sn % 4 == 0 && ((uintptr_t)L.x & 15) == 0 && L.h * L.w < (1ll << 30) && L.n < (1ll << 31)) {
    global_avg_cl4_kernel<<<(unsigned)L.n, 256, 0, stream>>>(L);
    PFB_CUDA(cudaGetLastError());
    return;
  }
  if (L.mode == 2 && L.oh == 1 && L.ow == 1 && L.sc == 1 && L.n < 65536) {
    dim3 grid((unsigned)ceil_div(L.c, 32), (unsigned)L.n, 1);
    global_avg_cl_kernel<<<grid, 1024, 0, stream>>>(L);
    PFB_CUDA(cudaGetLastError());
    return;
  }
  const long long rows = L.n * L.oh;
  const bool cl4 = L.mode != 2 && L.sc == 1 && L.osc == 1 && L.c % 4 == 0 && L.sw % 4 == 0 && L.sh % 4 == 0 &&
                   L.sn % 4 == 0 && L.osw % 4 == 0 && L.osh % 4 == 0 && L.osn % 4 == 0 &&
                   ((uintptr_t)L.x & 15) == 0 && (!L.y || ((uintptr_t)L.y & 15) == 0) &&
                   (!L.out_hi || ((uintptr_t)L.out_hi & 15) == 0) && (!L.out_lo || ((uintptr_t)L.out_lo & 15) == 0) &&
                   L.h * L.sh < (1ll << 31) && L.w * L.sw < (1ll << 31) && rows < (1ll << 31);
  if (cl4) {
    const long long inner = (L.c / 4) * L.ow;
    dim3 grid((unsigned)ceil_div(inner, 128), (unsigned)std::min<long long>(rows, 65535), 1);
    pool_cl_kernel<<<grid, 128, 0, stream>>>(L);
    PFB_CUDA(cudaGetLastError());
    return;
  }
  const long long inner = L.c * L.ow;
  dim3 grid((unsigned)ceil_div(inner, 256), (unsigned)std::min<long long>(rows, 65535), 1);
  pool_kernel<<<grid, 256, 0, stream>>>(L);
  PFB_CUDA(cudaGetLastError());
}

void launch_conv_input(const ConvInputLaunch& L, cudaStream_t stream) {
  PFB_CHECK_ARG(L.x && L.hi && (L.precision == PFC_PRECISION_BF16 || L.lo), "conv input: null pointer");
  PFB_CHECK_ARG(L.cp >= L.c && L.c > 0 && L.cp % 4 == 0, "conv input: padded channels must cover the channels");
  PFB_CHECK_ARG(((uintptr_t)L.hi & 15) == 0 && ((uintptr_t)L.lo & 15) == 0, "conv input: outputs must be 16-byte aligned");
  PFB_CHECK_ARG(L.hp == 0 || (L.hp >= L.h + L.ph && L.wp >= L.w + L.pw), "conv input: padded extent too small");
  PFB_CHECK_ARG(L.precision != PFC_PRECISION_BF16 || L.cp % 8 == 0, "conv input: bf16 channels come in groups of 8");
  PFB_CHECK_ARG(!L.deint || (L.hp > 0 && L.wp % 2 == 0), "conv input: de-interleaved rows need an even padded width");
  const long long total = L.n * (L.hp > 0 ? L.hp * L.wp : L.h * L.w);  // output pixels, one thread each
  if (total == 0) return;
  const unsigned g = grid_for(total, 256);
  const bool small = total * L.cp < (1ll << 30);  // element offsets and pixel + grid stride stay below 2^31
  if (L.precision == PFC_PRECISION_BF16) {
    if (small) conv_input_kernel<PFC_PRECISION_BF16, int><<<g, 256, 0, stream>>>(L);
    else conv_input_kernel<PFC_PRECISION_BF16, long long><<<g, 256, 0, stream>>>(L);
  } else {
    if (small) conv_input_kernel<PFC_PRECISION_TF32X3, int><<<g, 256, 0, stream>>>(L);
    else conv_input_kernel<PFC_PRECISION_TF32X3, long long><<<g, 256, 0, stream>>>(L);
  }
  PFB_CUDA(cudaGetLastError());
}

void launch_conv_weight(const ConvWeightLaunch& L, cudaStream_t stream) {
  PFB_CHECK_ARG(L.w && L.hi && (L.precision == PFC_PRECISION_BF16 || L.lo), "conv weight: null pointer");
  PFB_CHECK_ARG(L.cp >= L.c && (L.kwp == 0 || L.kwp >= L.kw) &&
                    L.kpad >= L.kh * (L.kwp > 0 ? L.kwp : L.kw) * L.cp,
                "conv weight: bad layout");
  const long long total = L.o * L.kpad;
  if (total == 0) return;
  if (L.precision == PFC_PRECISION_BF16) conv_weight_kernel<PFC_PRECISION_BF16><<<grid_for(total, 256), 256, 0, stream>>>(L);
  else conv_weight_kernel<PFC_PRECISION_TF32X3><<<grid_for(total, 256), 256, 0, stream>>>(L);
  PFB_CUDA(cudaGetLastError());
}

void launch_bn_fold(const BnFoldLaunch& L, cudaStream_t stream) {
  if (L.channels == 0) return;
  bn_fold_kernel<<<grid_for(L.channels, 256), 256, 0, stream>>>(L);
  PFB_CUDA(cudaGetLastError());
}

}  // namespace pfb
