// Activations applied in the GEMM epilogues, as PyFlame's CPU executor
// evaluates them (executor.cpp:392-416): 1 ReLU (NaN -> 0), 2 GELU in the tanh
// form, 3 sigmoid, 4 tanh, 5 SiLU; 0 none.  Full-precision expf/tanhf and
// IEEE division (these run once per output element, not per term).
#pragma once

namespace pfb {

template <int ACT>
__device__ __forceinline__ float act_apply(float v) {
  if constexpr (ACT == 1) return (0.f < v) ? v : 0.f;
  else if constexpr (ACT == 2) return 0.5f * v * (1.0f + tanhf(0.7978845608f * (v + 0.044715f * v * v * v)));
  else if constexpr (ACT == 3) return 1.0f / (1.0f + expf(-v));
  else if constexpr (ACT == 4) return tanhf(v);
  else if constexpr (ACT == 5) return v / (1.0f + expf(-v));
  else return v;
}

// The same with the code known only at run time.
__device__ __forceinline__ float act_apply_rt(int act, float v) {
  switch (act) {
    case 1: return act_apply<1>(v);
    case 2: return act_apply<2>(v);
    case 3: return act_apply<3>(v);
    case 4: return act_apply<4>(v);
    case 5: return act_apply<5>(v);
    default: return v;
  }
}

}  // namespace pfb
