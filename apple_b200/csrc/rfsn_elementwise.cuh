// rfsn_elementwise.cuh — element-wise steps of the decoder layer shared by several kernels.
#pragma once

#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include "rfsn_common.cuh"

namespace rfsn {

__device__ __forceinline__ float round_f16(float v) { return __half2float(__float2half_rn(v)); }

// The layer's tanh-approximate GELU (attention.py:137-138): 0.5 x (1 + tanh(0.7978845608 (x +
// 0.044715 x^3))) with every product, sum and the tanh computed in fp32 from fp16 operands and
// rounded to fp16 before the next operation, as the layer's fp16 expression is evaluated.
__device__ __forceinline__ uint16_t gelu_tanh_f16(uint16_t xh) {
  const float x = h2f(xh);
  const float x3 = round_f16(__fmul_rn(__fmul_rn(x, x), x));
  const float inner = round_f16(__fadd_rn(x, round_f16(__fmul_rn(0.044715f, x3))));
  const float t = round_f16(tanhf(round_f16(__fmul_rn(0.7978845608f, inner))));
  const float half_x = round_f16(__fmul_rn(0.5f, x));
  return f2h(__fmul_rn(half_x, round_f16(__fadd_rn(1.0f, t))));
}

}  // namespace rfsn
