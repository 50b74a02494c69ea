// Gated activations shared by the standalone kernels (fused.cu) and the GEMM epilogues that
// apply them to a gate_up output (tileops/fused.py:97-114, kernels
// tileops/backend/cuda/fused.py:17-43):
//   silu(x) = x * sigmoid(x),  gelu_tanh(x) = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
// Arithmetic in fp32; the activation is rounded to the tensor dtype before the multiply and the
// product rounded again, the two roundings of `act(a) * b` in the tensor dtype.
#pragma once

#include "common.cuh"

namespace tob {

enum Act : int { kSilu = 0, kGeluTanh = 1 };

template <int OP>
__device__ __forceinline__ float act_f32(float x) {
  if constexpr (OP == kSilu) {
    return x / (1.0f + expf(-x));
  } else {
    const float inner = 0.7978845608028654f * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.0f + tanhf(inner));
  }
}

template <typename T, int OP>
__device__ __forceinline__ T act_mul(T a, T b) {
  const T g = from_f32<T>(act_f32<OP>(to_f32<T>(a)));
  return from_f32<T>(to_f32<T>(g) * to_f32<T>(b));
}

}  // namespace tob
