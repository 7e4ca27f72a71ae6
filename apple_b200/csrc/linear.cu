// linear.cu — decode-shaped projections of RFSNDecoderLayerMLX
// (rfsn_v10_mlx_ane_complete.py:114-172): y[M x N] = x[M x K] . w[N x K]^T with
// M <= 32 rows (one token per sequence), fp16 in and out, fp32 accumulation.
//
// At decode the projections are weight streams: 32 activation rows against
// megabytes of weights, so the bound is HBM.  A CTA owns 32 output features and
// its 8 warps split K.  Each lane loads 16 contiguous bytes of a weight row and
// of an activation row per 32-wide k chunk; the mma's k order is free (the sum
// is the same for any permutation applied to both operands), so those 16 bytes
// feed two mma.m16n8k16 steps directly: k index 2q+e of the first step is
// element 8q+e of the chunk, 2q+8+e is element 8q+2+e, and the second step
// takes elements 8q+4.. and 8q+6...  Every 32-byte sector a warp touches is
// fully used.  The 8 partial sums are added in shared memory and rounded once
// to fp16, as a library GEMM with fp32 accumulation rounds its result.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "rfsn_api_internal.h"
#include "rfsn_attn_util.cuh"
#include "rfsn_common.cuh"

namespace rfsn {

constexpr int kLinWarps = 8;
constexpr int kLinBN = 32;  // output features per CTA (4 n8 tiles)

__device__ __forceinline__ uint4 ldg_nc16(const uint16_t* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// MT m16 tiles of rows (MT = 1: M <= 16; MT = 2: M <= 32).
template <int MT>
__global__ void __launch_bounds__(kLinWarps * 32) linear_small_m_kernel(const uint16_t* __restrict__ x,
                                                                        const uint16_t* __restrict__ w,
                                                                        uint16_t* __restrict__ y, int M, int K,
                                                                        int64_t ldx, int64_t ldy) {
  __shared__ float s_part[kLinWarps][16 * MT][kLinBN + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t n0 = (int64_t)blockIdx.x * kLinBN;
  const int kslice = K / kLinWarps;
  const int kb = warp * kslice;
  float acc[MT][4][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int t = 0; t < 4; ++t) acc[mt][t][0] = acc[mt][t][1] = acc[mt][t][2] = acc[mt][t][3] = 0.f;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll 2
  for (int kc = kb; kc < kb + kslice; kc += 32) {
    uint4 xa[2 * MT], wb[4];
#pragma unroll
    for (int i = 0; i < 2 * MT; ++i) {  // activation rows g + 8i (m16 tile i/2, half i%2)
      const int r = g + 8 * i;
      xa[i] = r < M ? ldg_nc16(x + (int64_t)r * ldx + kc + 8 * q) : zero;
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) wb[t] = ldg_nc16(w + (n0 + 8 * t + g) * (int64_t)K + kc + 8 * q);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const uint4 lo = xa[2 * mt], hi = xa[2 * mt + 1];
      const uint32_t a_first[4] = {lo.x, hi.x, lo.y, hi.y};   // chunk elements 8q+0..3
      const uint32_t a_second[4] = {lo.z, hi.z, lo.w, hi.w};  // chunk elements 8q+4..7
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        mma16816(acc[mt][t], a_first, wb[t].x, wb[t].y);
        mma16816(acc[mt][t], a_second, wb[t].z, wb[t].w);
      }
    }
  }
  // D fragment: rows 16mt + g (+8), features 8t + 2q (+1)
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int r = 16 * mt + g, cidx = 8 * t + 2 * q;
      s_part[warp][r][cidx] = acc[mt][t][0];
      s_part[warp][r][cidx + 1] = acc[mt][t][1];
      s_part[warp][r + 8][cidx] = acc[mt][t][2];
      s_part[warp][r + 8][cidx + 1] = acc[mt][t][3];
    }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 16 * MT * kLinBN; idx += blockDim.x) {
    const int r = idx / kLinBN, cidx = idx - r * kLinBN;
    if (r >= M) continue;
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kLinWarps; ++k) s += s_part[k][r][cidx];
    y[(int64_t)r * ldy + n0 + cidx] = f2h(s);
  }
}

}  // namespace rfsn

using namespace rfsn;

extern "C" int rfsn_linear_f16(const uint16_t* x, const uint16_t* w, uint16_t* y, int64_t M, int64_t N, int64_t K,
                               int64_t ldx, int64_t ldy, void* stream) {
  if (M < 0 || N < 0 || K < 0 || ldx < K || ldy < N) return RFSN_ERR_INVALID_ARGUMENT;
  if (M == 0 || N == 0) return RFSN_OK;
  if (!x || !w || !y) return RFSN_ERR_INVALID_ARGUMENT;
  // shapes this kernel serves: decode rows, whole 32-feature tiles, K split evenly into 32-wide chunks
  if (M > 32 || N % kLinBN || K % (kLinWarps * 32) || K == 0 || N / kLinBN > 0x7fffffff)
    return RFSN_ERR_UNSUPPORTED;
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) || (ldx & 7)) return RFSN_ERR_ALIGNMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(N / kLinBN));
  if (M <= 16)
    linear_small_m_kernel<1><<<grid, kLinWarps * 32, 0, s>>>(x, w, y, (int)M, (int)K, ldx, ldy);
  else
    linear_small_m_kernel<2><<<grid, kLinWarps * 32, 0, s>>>(x, w, y, (int)M, (int)K, ldx, ldy);
  return check_cuda(cudaGetLastError());
}
