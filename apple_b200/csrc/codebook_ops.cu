// codebook_ops.cu — affine low-bit quantization of codebooks (the reference's optional
// quantize_codebooks_for_ane path, quantization.py:36-89 and 159-175, 277-293).
//
// The reference quantizes each codebook matrix with MLX's mx.quantize (MLX 0.29.3,
// affine mode) and afterwards reads the codebooks back through mx.dequantize.  The
// published affine scheme, per group of `group` consecutive elements of a row:
//
//   alpha = max(w), beta = min(w), scale = (alpha - beta) / (2^bits - 1)
//   q = round((w - beta) / scale) clipped to [0, 2^bits - 1]   (round half to even)
//   dequantized w' = q * scale + beta
//
// all in fp32.  A group whose elements are all equal has scale 0: its codes are 0
// and w' = beta.  One warp per group; group <= 128.
#include <cuda_runtime.h>
#include <math.h>

#include "rfsn_api_internal.h"

namespace rfsn {

__global__ void affine_quantize_kernel(const float* __restrict__ w, int64_t groups, int group, int bits,
                                       uint8_t* __restrict__ q, float* __restrict__ scales,
                                       float* __restrict__ biases, float* __restrict__ deq) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const float nbins = (float)((1 << bits) - 1);
  for (int64_t g = gw; g < groups; g += nwarps) {
    const float* src = w + g * group;
    float mx = -INFINITY, mn = INFINITY;
    for (int i = lane; i < group; i += 32) {
      mx = fmaxf(mx, src[i]);
      mn = fminf(mn, src[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    }
    const float scale = __fdiv_rn(__fsub_rn(mx, mn), nbins);
    for (int i = lane; i < group; i += 32) {
      float c = 0.f;
      if (scale > 0.f) c = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(src[i], mn), scale)), 0.f), nbins);
      q[g * group + i] = (uint8_t)c;
      deq[g * group + i] = __fadd_rn(__fmul_rn(c, scale), mn);
    }
    if (lane == 0) {
      scales[g] = scale;
      biases[g] = mn;
    }
  }
}

}  // namespace rfsn

using namespace rfsn;

extern "C" int rfsn_affine_quantize_f32(const float* w, int64_t rows, int cols, int group, int bits, uint8_t* q,
                                        float* scales, float* biases, float* dequantized, void* stream) {
  if (rows < 0 || cols <= 0 || group <= 0 || group > 128 || cols % group || bits < 1 || bits > 8)
    return RFSN_ERR_INVALID_ARGUMENT;
  if (rows == 0) return RFSN_OK;
  if (!w || !q || !scales || !biases || !dequantized) return RFSN_ERR_INVALID_ARGUMENT;
  const int64_t groups = rows * (cols / group);
  int64_t blocks = (groups * 32 + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  affine_quantize_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      w, groups, group, bits, q, scales, biases, dequantized);
  return check_cuda(cudaGetLastError());
}
