// layer_ops.cu — fused element-wise steps of RFSNDecoderLayerMLX
// (rfsn_v10_mlx_ane_complete.py:114-172): RMSNorm and the tanh-approximate GELU.
//
// The layer evaluates both as chains of fp32/fp16 tensor operations; at decode
// sizes (a few rows of a few thousand features) every operation is a separate
// launch whose cost is its latency.  Here each is one kernel that keeps the
// same operation order and the same rounding points:
//
//   RMSNorm  y = fp16((x * rsqrt(mean(x^2) + eps)) * w), all in fp32 (the layer's
//            _RMSNorm; mlx.nn.RMSNorm).  The sum of squares is reduced in a
//            different order than a framework reduction, so y may differ from
//            such a chain by an fp16 rounding step where the mean differs in its
//            last fp32 bit.
//   GELU     attention.py:137-138, 0.5 * x * (1 + tanh(0.7978845608 * (x +
//            0.044715 * x^3))) evaluated operation by operation in fp16 as the
//            layer does: each product, sum and the tanh are computed in fp32 from
//            fp16 operands and rounded to fp16 before the next operation.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "rfsn_api_internal.h"
#include "rfsn_common.cuh"

namespace rfsn {

constexpr int kNormThreads = 256;

// fp16 a + b as the layer's fp16 tensor add rounds it (fp32 sum, one rounding)
__device__ __forceinline__ uint32_t hadd2_round(uint32_t a, uint32_t b) {
  const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&a));
  const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&b));
  const __half2 h = __floats2half2_rn(__fadd_rn(fa.x, fb.x), __fadd_rn(fa.y, fb.y));
  return *reinterpret_cast<const uint32_t*>(&h);
}

// One CTA per row.  Rows with dim % 8 == 0 and 16-byte aligned rows use 16-byte
// loads; any other row shape takes the scalar loop.  With `b` set, the row is
// first x + b (fp16), written to `sum` and normalised (the layer's residual add
// followed by its FFN RMSNorm); the row is re-read from `sum` by the thread
// that wrote it.
// (x and sum are not __restrict__: with b set the row is read back from sum, which
// this kernel writes, so those loads must not take the read-only path)
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const uint16_t* x, const uint16_t* __restrict__ b,
                                                               uint16_t* sum,
                                                               const float* __restrict__ w,
                                                               uint16_t* __restrict__ y, int dim, float eps,
                                                               int vec) {
  __shared__ float s_part[kNormThreads / 32];
  const int64_t row = blockIdx.x;
  const uint16_t* xr = x + row * dim;
  uint16_t* yr = y + row * dim;
  if (b) {  // residual add; the rest of the kernel reads the sum back
    const uint16_t* br = b + row * dim;
    uint16_t* sr = sum + row * dim;
    if (vec) {
      for (int i = threadIdx.x; i < dim / 8; i += blockDim.x) {
        const uint4 u = reinterpret_cast<const uint4*>(xr)[i];
        const uint4 v = reinterpret_cast<const uint4*>(br)[i];
        reinterpret_cast<uint4*>(sr)[i] =
            make_uint4(hadd2_round(u.x, v.x), hadd2_round(u.y, v.y), hadd2_round(u.z, v.z), hadd2_round(u.w, v.w));
      }
    } else {
      for (int i = threadIdx.x; i < dim; i += blockDim.x) sr[i] = f2h(__fadd_rn(h2f(xr[i]), h2f(br[i])));
    }
    xr = sr;  // each thread re-reads only the elements it wrote (same loop order)
  }
  float ss = 0.f;
  if (vec) {
    for (int i = threadIdx.x; i < dim / 8; i += blockDim.x) {
      const uint4 v = reinterpret_cast<const uint4*>(xr)[i];
      const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[k]));
        ss = __fmaf_rn(f.x, f.x, ss);
        ss = __fmaf_rn(f.y, f.y, ss);
      }
    }
  } else {
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
      const float f = h2f(xr[i]);
      ss = __fmaf_rn(f, f, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int k = 0; k < (int)(blockDim.x >> 5); ++k) tot += s_part[k];
  const float r = rsqrtf(__fadd_rn(__fmul_rn(tot, 1.0f / (float)dim), eps));  // mean as sum * (1/n)
  if (vec) {
    for (int i = threadIdx.x; i < dim / 8; i += blockDim.x) {
      const uint4 v = reinterpret_cast<const uint4*>(xr)[i];
      const float4 wa = reinterpret_cast<const float4*>(w)[2 * i];
      const float4 wb = reinterpret_cast<const float4*>(w)[2 * i + 1];
      const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
      uint32_t o4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[k]));
        const __half2 h = __floats2half2_rn(__fmul_rn(__fmul_rn(f.x, r), wv[2 * k]),
                                            __fmul_rn(__fmul_rn(f.y, r), wv[2 * k + 1]));
        o4[k] = *reinterpret_cast<const uint32_t*>(&h);
      }
      reinterpret_cast<uint4*>(yr)[i] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
    }
  } else {
    for (int i = threadIdx.x; i < dim; i += blockDim.x) yr[i] = f2h(__fmul_rn(__fmul_rn(h2f(xr[i]), r), w[i]));
  }
}

__device__ __forceinline__ float rh(float v) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ uint16_t gelu_tanh_f16(uint16_t xh) {
  const float x = h2f(xh);
  const float x3 = rh(__fmul_rn(__fmul_rn(x, x), x));
  const float inner = rh(__fadd_rn(x, rh(__fmul_rn(0.044715f, x3))));
  const float t = rh(tanhf(rh(__fmul_rn(0.7978845608f, inner))));
  const float half_x = rh(__fmul_rn(0.5f, x));
  return f2h(__fmul_rn(half_x, rh(__fadd_rn(1.0f, t))));
}

__global__ void gelu_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int64_t n, int vec) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n / 8; i += stride) {
      const uint4 v = reinterpret_cast<const uint4*>(x)[i];
      const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
      uint32_t o4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        o4[k] = (uint32_t)gelu_tanh_f16((uint16_t)(w4[k] & 0xffffu)) |
                ((uint32_t)gelu_tanh_f16((uint16_t)(w4[k] >> 16)) << 16);
      reinterpret_cast<uint4*>(y)[i] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
    }
  } else {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) y[i] = gelu_tanh_f16(x[i]);
  }
}

}  // namespace rfsn

using namespace rfsn;

extern "C" int rfsn_rmsnorm_f16(const uint16_t* x, const float* weight, uint16_t* y, int64_t rows, int dim,
                                float eps, void* stream) {
  if (rows < 0 || dim <= 0 || (rows > 0 && (!x || !weight || !y))) return RFSN_ERR_INVALID_ARGUMENT;
  if (rows > 0x7fffffff) return RFSN_ERR_UNSUPPORTED;
  if (rows == 0) return RFSN_OK;
  const int vec = dim % 8 == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(weight) & 15) == 0;
  rmsnorm_kernel<<<(unsigned)rows, kNormThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, nullptr, nullptr, weight, y, dim, eps, vec);
  return check_cuda(cudaGetLastError());
}

extern "C" int rfsn_add_rmsnorm_f16(const uint16_t* x, const uint16_t* b, uint16_t* sum, const float* weight,
                                    uint16_t* y, int64_t rows, int dim, float eps, void* stream) {
  if (rows < 0 || dim <= 0 || (rows > 0 && (!x || !b || !sum || !weight || !y))) return RFSN_ERR_INVALID_ARGUMENT;
  if (rows > 0x7fffffff) return RFSN_ERR_UNSUPPORTED;
  if (rows == 0) return RFSN_OK;
  const uintptr_t ptrs = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(b) |
                         reinterpret_cast<uintptr_t>(sum) | reinterpret_cast<uintptr_t>(y) |
                         reinterpret_cast<uintptr_t>(weight);
  const int vec = dim % 8 == 0 && (ptrs & 15) == 0;
  rmsnorm_kernel<<<(unsigned)rows, kNormThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, b, sum, weight, y,
                                                                                            dim, eps, vec);
  return check_cuda(cudaGetLastError());
}

extern "C" int rfsn_gelu_tanh_f16(const uint16_t* x, uint16_t* y, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!x || !y))) return RFSN_ERR_INVALID_ARGUMENT;
  if (n == 0) return RFSN_OK;
  const int vec = n % 8 == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  const int64_t work = vec ? n / 8 : n;
  int64_t blocks = (work + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  gelu_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, y, n, vec);
  return check_cuda(cudaGetLastError());
}
