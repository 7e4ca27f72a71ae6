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
#include "rfsn_elementwise.cuh"

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
// kLlama: the Llama adapter's form (llama32_adapter.py:497-500): x / sqrt(mean + eps), times an
// fp16 weight (W = uint16_t) instead of x * rsqrt(mean + eps) times an fp32 weight.
__device__ __forceinline__ float wload(const float* w, int i) { return w[i]; }
__device__ __forceinline__ float wload(const uint16_t* w, int i) { return h2f(w[i]); }

template <bool kLlama, typename W>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const uint16_t* x, const uint16_t* __restrict__ b,
                                                               uint16_t* sum,
                                                               const W* __restrict__ w,
                                                               uint16_t* __restrict__ y, int dim, float eps,
                                                               int vec) {
  __shared__ float s_part[kNormThreads / 32];
  griddep_launch();  // a projection launched after this kernel may start streaming its weights
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
  const float var = __fadd_rn(__fmul_rn(tot, 1.0f / (float)dim), eps);  // mean as sum * (1/n)
  const float r = kLlama ? __fsqrt_rn(var) : rsqrtf(var);
  if (kLlama) {  // fp32 x / sqrt(var) * w, rounded once to fp16 per element
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
      yr[i] = f2h(__fmul_rn(__fdiv_rn(h2f(xr[i]), r), wload(w, i)));
    return;
  }
  if (vec) {
    for (int i = threadIdx.x; i < dim / 8; i += blockDim.x) {
      const uint4 v = reinterpret_cast<const uint4*>(xr)[i];
      const float4 wa = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(w))[2 * i];
      const float4 wb = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(w))[2 * i + 1];
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
    for (int i = threadIdx.x; i < dim; i += blockDim.x) yr[i] = f2h(__fmul_rn(__fmul_rn(h2f(xr[i]), r), wload(w, i)));
  }
}

// Rotary embedding of the Llama adapter (llama32_adapter.py:555-568): y = fp16(x * cos +
// rotate_half(x) * sin) in fp32 with each product and the sum rounded separately, for
// x [batch][seq][heads][dim] (strides in elements, dim contiguous) and fp16 tables [seq][dim].
// rotate_half(x)[d] = -x[d + dim/2] for d < dim/2, x[d - dim/2] otherwise.  y may alias x
// (each thread reads its pair before writing it).
__global__ void rope_kernel(const uint16_t* x, uint16_t* y, const uint16_t* __restrict__ cosv,
                            const uint16_t* __restrict__ sinv, int64_t batch, int seq, int heads, int dim,
                            int64_t sb, int64_t ss, int64_t sh, int64_t yb, int64_t ys, int64_t yh) {
  const int half = dim / 2;
  const int64_t n = batch * seq * heads * half;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % half);
    int64_t r = i / half;
    const int h = (int)(r % heads);
    r /= heads;
    const int s = (int)(r % seq);
    const int64_t b = r / seq;
    const uint16_t* xr = x + b * sb + s * ss + h * sh;
    uint16_t* yr = y + b * yb + s * ys + h * yh;
    const float lo = h2f(xr[d]), hi = h2f(xr[d + half]);
    const float c0 = h2f(cosv[(int64_t)s * dim + d]), s0 = h2f(sinv[(int64_t)s * dim + d]);
    const float c1 = h2f(cosv[(int64_t)s * dim + d + half]), s1 = h2f(sinv[(int64_t)s * dim + d + half]);
    yr[d] = f2h(__fadd_rn(__fmul_rn(lo, c0), __fmul_rn(-hi, s0)));
    yr[d + half] = f2h(__fadd_rn(__fmul_rn(hi, c1), __fmul_rn(lo, s1)));
  }
}

// SwiGLU of the Llama adapter (llama32_adapter.py:502-504, 584-589): a = fp16(g * sigmoid(g))
// in fp32 with sigmoid(g) = 1 / (1 + exp(-g)), then y = fp16(a * u).
__global__ void silu_mul_kernel(const uint16_t* __restrict__ g, const uint16_t* __restrict__ u,
                                uint16_t* __restrict__ y, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float gv = h2f(g[i]);
    const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
    const float a = h2f(f2h(__fmul_rn(gv, sg)));
    y[i] = f2h(__fmul_rn(a, h2f(u[i])));
  }
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
  rmsnorm_kernel<false, float><<<(unsigned)rows, kNormThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
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
  rmsnorm_kernel<false, float><<<(unsigned)rows, kNormThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, b, sum, weight, y, dim, eps, vec);
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

extern "C" int rfsn_llama_rmsnorm_f16(const uint16_t* x, const uint16_t* b, uint16_t* sum, const uint16_t* weight,
                                      uint16_t* y, int64_t rows, int dim, float eps, void* stream) {
  if (rows < 0 || dim <= 0 || (rows > 0 && (!x || !weight || !y || (b && !sum)))) return RFSN_ERR_INVALID_ARGUMENT;
  if (rows > 0x7fffffff) return RFSN_ERR_UNSUPPORTED;
  if (rows == 0) return RFSN_OK;
  const uintptr_t ptrs = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(b) |
                         reinterpret_cast<uintptr_t>(sum);
  const int vec = dim % 8 == 0 && (ptrs & 15) == 0;  // the residual add's loads
  rmsnorm_kernel<true, uint16_t><<<(unsigned)rows, kNormThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, b, sum, weight, y, dim, eps, vec);
  return check_cuda(cudaGetLastError());
}

extern "C" int rfsn_rope_f16(const uint16_t* x, int64_t stride_b, int64_t stride_s, int64_t stride_h, uint16_t* y,
                             int64_t y_stride_b, int64_t y_stride_s, int64_t y_stride_h, const uint16_t* cos_table,
                             const uint16_t* sin_table, int64_t batch, int seq, int heads, int dim, void* stream) {
  if (batch < 0 || seq < 0 || heads < 0 || dim <= 0 || dim % 2) return RFSN_ERR_INVALID_ARGUMENT;
  const int64_t n = batch * seq * heads * (dim / 2);
  if (n == 0) return RFSN_OK;
  if (!x || !y || !cos_table || !sin_table) return RFSN_ERR_INVALID_ARGUMENT;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  rope_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, y, cos_table, sin_table, batch, seq, heads, dim, stride_b, stride_s, stride_h, y_stride_b, y_stride_s,
      y_stride_h);
  return check_cuda(cudaGetLastError());
}

extern "C" int rfsn_silu_mul_f16(const uint16_t* gate, const uint16_t* up, uint16_t* y, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!gate || !up || !y))) return RFSN_ERR_INVALID_ARGUMENT;
  if (n == 0) return RFSN_OK;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  silu_mul_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(gate, up, y, n);
  return check_cuda(cudaGetLastError());
}
