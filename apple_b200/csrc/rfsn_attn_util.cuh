// rfsn_attn_util.cuh — register-level building blocks of the fused decode kernel.
//
// * mma16816: one mma.sync.m16n8k16 (f16 x f16 -> f32 accumulate).  Products of
//   fp16 values are exact in fp32, so scores equal fp32 dot products up to the
//   accumulation order.
// * mma16808: one mma.sync.m16n8k8 (f16 x f16 -> f32 accumulate), used for P.V.
// * split_h2: two fp32 probabilities as fp16 hi + lo pairs (p = hi + lo to about
//   22 bits), so P.V on tensor cores keeps near-fp32 weights.
// * rvq_add8: fp16 RVQ correction of 8 dims (one layer: fp16 row; several:
//   fp16 of the fp32 sum of rows, as rfsn_decode.cuh::recon8), added in fp16.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace rfsn {

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma16808(float c[4], uint32_t a0, uint32_t a1, uint32_t b) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(b));
}

// byte permute: result byte i = byte (sel >> 4i) & 7 of the 8-byte value {b, a}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// (p0, p1) -> hi = fp16x2 of (p0, p1), lo = fp16x2 of the remainders p - float(hi)
__device__ __forceinline__ void split_h2(float p0, float p1, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(p0, p1);
  const float2 hf = __half22float2(h);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = pack_h2(p0 - hf.x, p1 - hf.y);
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
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

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  const __half2 s = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&s);
}

__device__ __forceinline__ uint32_t hadd2_u32(uint32_t a, uint32_t b) {
  const __half2 s = __hadd2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&s);
}

// RVQ correction of dims [d0, d0+8) added to o (fp16 words), layers summed in
// fp32.  Codes are clamped to Kr - 1 so stray bytes never index past the codebook.
template <int D>
__device__ __forceinline__ void rvq_add8(const uint16_t* cb, int L, int Kr, int rvq_u16, const unsigned char* rc,
                                         int d0, uint32_t* o) {
  const uint32_t kmax = (uint32_t)Kr - 1u;
  const uint32_t c0 = min(rvq_u16 ? (uint32_t)*reinterpret_cast<const uint16_t*>(rc) : (uint32_t)rc[0], kmax);
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
    const uint32_t c = min(rvq_u16 ? (uint32_t)reinterpret_cast<const uint16_t*>(rc)[l] : (uint32_t)rc[l], kmax);
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

}  // namespace rfsn
