// rfsn_attn_util.cuh — register-level building blocks of the fused decode kernel.
//
// * mma16816: one mma.sync.m16n8k16 (f16 x f16 -> f32 accumulate).  Products of
//   fp16 values are exact in fp32, so scores equal fp32 dot products up to the
//   accumulation order.
// * split_h2: x = hi + lo with hi = fp16(x), lo = fp16(x - hi); feeding both
//   halves through an MMA with 0/1 weights sums fp32 values across lanes with
//   ~2^-22 relative error.
// * ffma2: two independent round-to-nearest fp32 FMAs in one fma.rn.f32x2.
// * recon_lane: exact fp16 reconstruction of one lane's dims of one token from
//   shared-memory codebooks (same arithmetic as rfsn_decode.cuh::recon8:
//   fp16 PQ centroid + fp16(fp32 sum of RVQ rows), fp16 add), specialised for
//   4- and 8-dim subspaces.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace rfsn {

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void split_h2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 hf = __half22float2(h);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = pack_h2(a - hf.x, b - hf.y);
}

__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void ffma2(float& a0, float& a1, float p, float x0, float x1) {
  asm("{\n\t.reg .b64 A, P, X;\n\t"
      "mov.b64 A, {%0, %1};\n\t"
      "mov.b64 P, {%2, %2};\n\t"
      "mov.b64 X, {%3, %4};\n\t"
      "fma.rn.f32x2 A, P, X, A;\n\t"
      "mov.b64 {%0, %1}, A;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(p), "f"(x0), "f"(x1));
}

__device__ __forceinline__ uint32_t ldg_u32(const uint16_t* p) { return __ldg(reinterpret_cast<const unsigned int*>(p)); }

template <int DPL>
__device__ __forceinline__ void load_dense(const uint16_t* src, uint32_t* w) {
#pragma unroll
  for (int g8 = 0; g8 < DPL / 8; ++g8) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + 8 * g8);
    w[4 * g8] = v.x; w[4 * g8 + 1] = v.y; w[4 * g8 + 2] = v.z; w[4 * g8 + 3] = v.w;
  }
}

template <int RMAX>
__device__ __forceinline__ void load_row(const float* src, float* out) {
  if constexpr (RMAX == 1) {
    out[0] = src[0];
  } else if constexpr (RMAX == 2) {
    const float2 v = *reinterpret_cast<const float2*>(src);
    out[0] = v.x; out[1] = v.y;
  } else {
#pragma unroll
    for (int i = 0; i < RMAX / 4; ++i) {
      const float4 v = *reinterpret_cast<const float4*>(src + 4 * i);
      out[4 * i] = v.x; out[4 * i + 1] = v.y; out[4 * i + 2] = v.z; out[4 * i + 3] = v.w;
    }
  }
}

template <int RMAX>
__device__ __forceinline__ void store_row(float* dst, const float* v) {
  if constexpr (RMAX == 1) {
    dst[0] = v[0];
  } else if constexpr (RMAX == 2) {
    *reinterpret_cast<float2*>(dst) = make_float2(v[0], v[1]);
  } else {
#pragma unroll
    for (int i = 0; i < RMAX / 4; ++i)
      *reinterpret_cast<float4*>(dst + 4 * i) = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
}

__device__ __forceinline__ uint32_t hadd2_u32(uint32_t a, uint32_t b) {
  const __half2 s = __hadd2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&s);
}

// PQ centroids of dims [d0, d0+8) (fp16, 4 words).  DS: 4 or 8 specialised; 0 = runtime ds.
template <int DS>
__device__ __forceinline__ void pq8(const uint16_t* cb, int K, int ds, const unsigned char* codes, int d0,
                                    uint32_t* o) {
  if constexpr (DS == 4) {
    const int m = d0 >> 2;
    const uint32_t c01 = *reinterpret_cast<const uint16_t*>(codes + m);
    const uint2 a = *reinterpret_cast<const uint2*>(cb + (((uint32_t)m * K + (c01 & 0xffu)) << 2));
    const uint2 b = *reinterpret_cast<const uint2*>(cb + (((uint32_t)(m + 1) * K + (c01 >> 8)) << 2));
    o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
  } else if constexpr (DS == 8) {
    const int m = d0 >> 3;
    const uint4 a = *reinterpret_cast<const uint4*>(cb + (((uint32_t)m * K + codes[m]) << 3));
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
  } else {
    if (ds >= 8) {
      const int m = d0 / ds;
      const int off = d0 - m * ds;
      const uint4 a = *reinterpret_cast<const uint4*>(cb + ((uint32_t)m * K + codes[m]) * ds + off);
      o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    } else if (ds == 4) {
      const int m = d0 >> 2;
      const uint2 a = *reinterpret_cast<const uint2*>(cb + (((uint32_t)m * K + codes[m]) << 2));
      const uint2 b = *reinterpret_cast<const uint2*>(cb + (((uint32_t)(m + 1) * K + codes[m + 1]) << 2));
      o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
    } else if (ds == 2) {
      const int m = d0 >> 1;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        o[i] = *reinterpret_cast<const uint32_t*>(cb + (((uint32_t)(m + i) * K + codes[m + i]) << 1));
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t lo = cb[(uint32_t)(d0 + 2 * i) * K + codes[d0 + 2 * i]];
        const uint32_t hi = cb[(uint32_t)(d0 + 2 * i + 1) * K + codes[d0 + 2 * i + 1]];
        o[i] = lo | (hi << 16);
      }
    }
  }
}

// RVQ correction of dims [d0, d0+8) added to o (fp16 words), layers summed in fp32.
template <int D>
__device__ __forceinline__ void rvq_add8(const uint16_t* cb, int L, int Kr, int rvq_u16, const unsigned char* rc,
                                         int d0, uint32_t* o) {
  const uint32_t c0 = rvq_u16 ? *reinterpret_cast<const uint16_t*>(rc) : rc[0];
  const uint4 r0 = *reinterpret_cast<const uint4*>(cb + c0 * D + d0);
  if (L == 1) {
    o[0] = hadd2_u32(o[0], r0.x); o[1] = hadd2_u32(o[1], r0.y);
    o[2] = hadd2_u32(o[2], r0.z); o[3] = hadd2_u32(o[3], r0.w);
    return;
  }
  float a[8];
  {
    const uint32_t w4[4] = {r0.x, r0.y, r0.z, r0.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
      a[2 * i] = 0.0f + f.x;
      a[2 * i + 1] = 0.0f + f.y;
    }
  }
  for (int l = 1; l < L; ++l) {
    const uint32_t c = rvq_u16 ? reinterpret_cast<const uint16_t*>(rc)[l] : rc[l];
    const uint4 r = *reinterpret_cast<const uint4*>(cb + ((uint32_t)l * Kr + c) * D + d0);
    const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
      a[2 * i] = __fadd_rn(a[2 * i], f.x);
      a[2 * i + 1] = __fadd_rn(a[2 * i + 1], f.y);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = hadd2_u32(o[i], pack_h2(a[2 * i], a[2 * i + 1]));
}

// Exact reconstruction of one lane's dims [dim0, dim0 + D/8) of a token.  The
// RVQ codebook is read from shared memory when it was staged (rvq_smem) and
// from global memory (L1/L2) otherwise.
template <int D, int DS>
__device__ __forceinline__ void recon_lane(const uint16_t* pq_cb, const uint16_t* rvq_s, const uint16_t* rvq_g,
                                           int rvq_smem, int K, int ds, int L, int Kr, int rvq_u16,
                                           const unsigned char* codes, const unsigned char* rcodes, bool act,
                                           int dim0, uint32_t* w) {
  constexpr int DPL = D / 8;
#pragma unroll
  for (int g8 = 0; g8 < DPL / 8; ++g8) pq8<DS>(pq_cb, K, ds, codes, dim0 + 8 * g8, w + 4 * g8);
  if (L > 0 && act) {
    if (rvq_smem) {
#pragma unroll
      for (int g8 = 0; g8 < DPL / 8; ++g8) rvq_add8<D>(rvq_s, L, Kr, rvq_u16, rcodes, dim0 + 8 * g8, w + 4 * g8);
    } else {
#pragma unroll
      for (int g8 = 0; g8 < DPL / 8; ++g8) rvq_add8<D>(rvq_g, L, Kr, rvq_u16, rcodes, dim0 + 8 * g8, w + 4 * g8);
    }
  }
}

}  // namespace rfsn
