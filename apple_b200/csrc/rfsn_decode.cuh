// rfsn_decode.cuh — exact reconstruction of 8 consecutive dims of one token.
//
// value = fp16( pq_decode + fp16( sum_l rvq_l ) )      (fp16 add, round to nearest even)
//
// exactly as the reference composes HybridQuantizerMLX.decode
// (quantization.py:310-319): the PQ centroids are fp16 (quantization.py:146-157),
// the RVQ correction is an fp32 sum over layers cast to fp16
// (quantization.py:266-272), inactive tokens get a zero correction (:261), and
// base + correction is an fp16 add (:319).  The top-S sparse residual (an
// extension) is added separately by the callers, in fp32.
#pragma once

#include "rfsn_common.cuh"

namespace rfsn {

struct QzView {
  const uint16_t* pq_cb;   // fp16 [M][K][ds] (shared or global memory)
  const uint16_t* rvq_cb;  // fp16 [L][Kr][D]
  int M, K, ds, L, Kr, D, S;
  int rvq_u16;
};

__device__ __forceinline__ uint32_t load_u32(const uint16_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// PQ part: dims [d0, d0 + 8) of a token whose M codes start at `codes`.
__device__ __forceinline__ void pq_gather8(const QzView& q, const uint8_t* codes, int d0, uint32_t out[4]) {
  const int ds = q.ds;
  if (ds >= 8) {
    const int m = d0 / ds;
    const int off = d0 - m * ds;
    const uint4 v = *reinterpret_cast<const uint4*>(q.pq_cb + ((size_t)(m * q.K + codes[m]) * ds + off));
    out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
  } else if (ds == 4) {
    const int m = d0 >> 2;
    const uint2 a = *reinterpret_cast<const uint2*>(q.pq_cb + ((size_t)(m * q.K + codes[m]) << 2));
    const uint2 b = *reinterpret_cast<const uint2*>(q.pq_cb + ((size_t)((m + 1) * q.K + codes[m + 1]) << 2));
    out[0] = a.x; out[1] = a.y; out[2] = b.x; out[3] = b.y;
  } else if (ds == 2) {
    const int m = d0 >> 1;
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = load_u32(q.pq_cb + ((size_t)((m + i) * q.K + codes[m + i]) << 1));
  } else {  // ds == 1
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = q.pq_cb[(size_t)(d0 + 2 * i) * q.K + codes[d0 + 2 * i]];
      const uint32_t hi = q.pq_cb[(size_t)(d0 + 2 * i + 1) * q.K + codes[d0 + 2 * i + 1]];
      out[i] = lo | (hi << 16);
    }
  }
}

__device__ __forceinline__ int rvq_code(const QzView& q, const void* codes, int l) {
  return q.rvq_u16 ? (int)reinterpret_cast<const uint16_t*>(codes)[l] : (int)reinterpret_cast<const uint8_t*>(codes)[l];
}

// fp16 RVQ correction for dims [d0, d0 + 8): one layer is the fp16 row itself,
// several layers are summed in fp32 in layer order and rounded once.
__device__ __forceinline__ void rvq_gather8(const QzView& q, const void* codes, int d0, uint32_t out[4]) {
  const int c0 = rvq_code(q, codes, 0);
  const uint4 r0 = *reinterpret_cast<const uint4*>(q.rvq_cb + ((size_t)c0 * q.D + d0));
  if (q.L == 1) {
    out[0] = r0.x; out[1] = r0.y; out[2] = r0.z; out[3] = r0.w;
    return;
  }
  float acc[8];
  {
    const uint32_t w[4] = {r0.x, r0.y, r0.z, r0.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      acc[2 * i] = 0.0f + f.x;
      acc[2 * i + 1] = 0.0f + f.y;
    }
  }
  for (int l = 1; l < q.L; ++l) {
    const int c = rvq_code(q, codes, l);
    const uint4 r = *reinterpret_cast<const uint4*>(q.rvq_cb + (((size_t)l * q.Kr + c) * q.D + d0));
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      acc[2 * i] = __fadd_rn(acc[2 * i], f.x);
      acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], f.y);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 h = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
    out[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
}

// Full exact reconstruction of dims [d0, d0+8) as 4 packed half2 words.
__device__ __forceinline__ void recon8(const QzView& q, const uint8_t* pq_codes, const void* rvq_codes, bool active,
                                       int d0, uint32_t out[4]) {
  pq_gather8(q, pq_codes, d0, out);
  if (q.L > 0 && active) {
    uint32_t c[4];
    rvq_gather8(q, rvq_codes, d0, c);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 s = __hadd2(*reinterpret_cast<const __half2*>(&out[i]), *reinterpret_cast<const __half2*>(&c[i]));
      out[i] = *reinterpret_cast<const uint32_t*>(&s);
    }
  }
}

__device__ __forceinline__ void unpack8(const uint32_t w[4], float f[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

}  // namespace rfsn
