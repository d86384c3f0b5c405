// Bias + activation of the tensor provider (reference runtime/tensor.cpp:79-115), shared
// by the standalone bias/activation kernel and the GEMM epilogues that fuse it, so a
// fused result equals matmul followed by bias/activation bit for bit.
#pragma once
#include <cstdint>

namespace pb {

// Tanh-form GELU with FP32 constants, in the reference's order of operations.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float cube = __fmul_rn(__fmul_rn(x, x), x);
  const float inner = __fadd_rn(x, __fmul_rn(0.044715f, cube));
  const float t = tanhf(__fmul_rn(0.7978845608028654f, inner));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}

// activation 0: none; 1: ReLU (values that compare below zero become +0.0, NaN and
// -0.0 pass through); 2: tanh-form GELU.
__device__ __forceinline__ float activate(float v, uint32_t activation) {
  if (activation == 1u && v < 0.0f)
    return 0.0f;
  if (activation == 2u)
    return gelu_tanh(v);
  return v;
}

// out = activate(fl(v + bias[column])) (no bias: activate(v)).
__device__ __forceinline__ float bias_activate(float v, const float *bias, int64_t column, uint32_t activation) {
  if (bias)
    v = __fadd_rn(v, bias[column]);
  return activate(v, activation);
}

} // namespace pb
