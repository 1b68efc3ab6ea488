// The 3xTF32 operand split, shared by every kernel that writes tensor-core
// operands (prepare, im2col, channels-last conv input, GEMM and pooling
// epilogues), so that an operand is bit-identical whichever kernel wrote it.
#pragma once

#include <cuda_runtime.h>

namespace pfb {

// hi keeps the sign, exponent and top 10 mantissa bits; lo is the exact
// remainder.  Non-finite values go entirely into hi (NaN canonicalised).
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  if (!isfinite(x)) {
    hi = isnan(x) ? __int_as_float(0x7fc00000) : x;
    lo = 0.f;
    return;
  }
  hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  lo = x - hi;
}

}  // namespace pfb
