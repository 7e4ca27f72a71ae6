// encode_tc.cu — spill encoder with nearest-centroid dot products on tensor cores.
//
// Same results as encode.cu's per-thread encoder (HybridQuantizerMLX.encode,
// quantization.py:124-144 and 206-252, plus the top-S sparse extension) for
// D = 64, 4- or 8-dim PQ subspaces, K <= 256 PQ centroids, at most one RVQ
// layer of Kr <= 256 rows (uint8 codes).  A warp encodes 16 vectors at a time:
//
//   PQ   per subspace m: mma.m16n8k8 gives x_m . c for 16 vectors x 8 centroids
//        (4-dim subspaces: the other half of k is zero in B); the epilogue forms
//        d = (|x_m|^2 - 2 x_m.c) + |c|^2 in fp32 exactly as the reference does
//        and keeps the first minimum (four independent chains per lane, merged
//        by distance then index, then across the lane quad by shuffles).
//   RVQ  residual r = fp16(x - c) (one rounding of the exact difference), norm
//        gate sqrt(sum r^2) > threshold, then mma.m16n8k16 over the 64 dims for
//        r . R[c] and the same epilogue.
//   sparse / stores: one lane per vector, CUDA cores.
//
// Small batches (a decode step appends one token per row: a few groups) run in
// split mode: the M warps of a group search one subspace each into the group
// leader's tiles, then the leader finishes the group, so the serial PQ search
// per warp is 1/M as long.  Large batches keep one warp per group.
//
// Products of fp16 values are exact in fp32, so d differs from the reference
// only through the dot products' summation order: codes can differ only where
// two candidates tie to fp32 rounding.  Operand fragments are read straight
// from shared memory with 32-bit loads; the x tile, residual tile and RVQ
// codebook rows are stored with their 16-byte chunks XOR-swizzled by row, so
// the 8 rows read by one load instruction fall in distinct banks.
#include <cuda_runtime.h>

#include "rfsn_api_internal.h"
#include "rfsn_attn_util.cuh"
#include "rfsn_common.cuh"
#include "rfsn_encode_tc.h"

namespace rfsn {

constexpr int kTcWarps = 16;  // warps per CTA (one CTA per SM)
constexpr int kTcD = 64;

struct EncTcParams {
  const uint16_t* x;
  const uint16_t* x_v;  // K and V in one launch: groups [ngk, 2 ngk) encode x_v into the V fields
  int64_t ngk;          // 16-vector groups of x
  int64_t batch, tokens, heads, sb, st, sh, nvec;
  uint8_t* data;
  BlockLayout lay;
  int kv;
  int64_t cap, rows, slot, first;
  uint16_t* residual_out;
  const uint16_t* pq_cb;
  const uint16_t* rvq_cb;
  int M, K, L, Kr, S;
  float thr;
  int split;  // warps per 16-vector group: 1, or M (one warp per PQ subspace, small batches)
  int smem_pq, smem_pqcc, smem_rvq, smem_rcc, smem_warp, warp_bytes;
};

__device__ __forceinline__ void mma1688(float c[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// 16-byte chunk q of row i of a swizzled [rows][64] fp16 tile (128 B rows).
__device__ __forceinline__ int swz(int i, int q) { return i * 8 + (q ^ (i & 7)); }

// Two candidates' distances (x_sq - 2 dot) + c_sq with one paired fma.rn.f32x2 and
// add.rn.f32x2: each element is rounded exactly as __fadd_rn(__fmaf_rn(-2, dot,
// x_sq), c_sq) rounds it, in half the instructions.
__device__ __forceinline__ void dist2(float& d0, float& d1, float dot0, float dot1, float xsq, float csq0,
                                     float csq1) {
  asm("{\n\t.reg .b64 C, M, X, D, E;\n\t"
      "mov.b64 C, {%2, %3};\n\t"
      "mov.b64 M, {%4, %4};\n\t"
      "mov.b64 X, {%5, %5};\n\t"
      "fma.rn.f32x2 D, M, C, X;\n\t"
      "mov.b64 E, {%6, %7};\n\t"
      "add.rn.f32x2 D, D, E;\n\t"
      "mov.b64 {%0, %1}, D;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(dot0), "f"(dot1), "f"(-2.f), "f"(xsq), "f"(csq0), "f"(csq1));
}

// Running first-minimum: take (d, idx) if strictly smaller.
__device__ __forceinline__ void take_min(float d, int idx, float& best, int& bi) {
  const bool p = d < best;
  best = p ? d : best;
  bi = p ? idx : bi;
}

// Merge two first-minima of disjoint index sets: smaller distance, then smaller index.
__device__ __forceinline__ void merge_min(float& best, int& bi, float d2, int i2) {
  const bool p = d2 < best || (d2 == best && i2 < bi);
  best = p ? d2 : best;
  bi = p ? i2 : bi;
}

// Lane-quad reduction (lanes 4r .. 4r+3 hold candidates for the same row).
__device__ __forceinline__ void quad_min(float& best, int& bi) {
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    const float d2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    merge_min(best, bi, d2, i2);
  }
}

// Token v = (b, t, h) of the [batch, tokens, heads] vectors; nvec < 2^31 (checked at
// launch), so 32-bit division suffices.
__device__ __forceinline__ int64_t vec_offset(const EncTcParams& p, uint32_t v) {
  const uint32_t heads = (uint32_t)p.heads, tokens = (uint32_t)p.tokens;
  const uint32_t bt = v / heads, h = v - bt * heads;
  const uint32_t b = bt / tokens, t = bt - b * tokens;
  return (int64_t)b * p.sb + (int64_t)t * p.st + (int64_t)h * p.sh;
}

// The four 16-byte chunks lane `lane` holds of group gg's x tile: rows (lane >> 3) + 4 s,
// chunk lane & 7; zero rows past the end.
__device__ __forceinline__ void fetch_x(const EncTcParams& p, int64_t gg, int lane, uint4 out[4]) {
  const bool isv = p.x_v != nullptr && gg >= p.ngk;
  const int64_t g = isv ? gg - p.ngk : gg;
  const uint16_t* xs = isv ? p.x_v : p.x;
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const int64_t v = g * 16 + (lane >> 3) + 4 * s;
    out[s] = make_uint4(0u, 0u, 0u, 0u);
    if (v < p.nvec) out[s] = __ldg(reinterpret_cast<const uint4*>(xs + vec_offset(p, (uint32_t)v)) + (lane & 7));
  }
}

template <int DS>
__global__ void __launch_bounds__(kTcWarps * 32, 1) encode_tc_kernel(const __grid_constant__ EncTcParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int M = kTcD / DS;
  uint16_t* s_pq = reinterpret_cast<uint16_t*>(smem + p.smem_pq);     // [M][K][DS] (global layout)
  float* s_pqcc = reinterpret_cast<float*>(smem + p.smem_pqcc);       // [M][K]
  uint4* s_rvq = reinterpret_cast<uint4*>(smem + p.smem_rvq);         // [Kr][8 chunks] swizzled
  float* s_rcc = reinterpret_cast<float*>(smem + p.smem_rcc);         // [Kr]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nthr = blockDim.x;
  const int K = p.K, Kr = p.Kr;

  const int split = p.split;
  const int gpc = (nthr >> 5) / split;  // groups per CTA and round
  const int gslot = warp / split, part = warp - gslot * split;
  const bool lead = part == 0;

  const int64_t ngroups = p.x_v ? 2 * p.ngk : p.ngk;
  // ---- stage codebooks and their squared norms (sequential fp32 sums) ----
  uint4 xpre[4];  // split mode: the leader's x rows, requested before the codebook staging
  if (split > 1) {
    // Split mode runs one round per CTA.  The leaders request their x rows first, so
    // that load's latency overlaps the staging.  Warp `part` of the first group then
    // stages PQ subspace `part` and sums its norms from the registers it loaded; the
    // barrier before the search publishes every slice to every warp (the leader's
    // residual step reads them after the barrier that follows the search).
    const int64_t gg0 = (int64_t)blockIdx.x * gpc + gslot;
    if (lead && gg0 < ngroups) fetch_x(p, gg0, lane, xpre);
    if (gslot == 0) {
      // 16-byte chunks of the slice: one 8-dim or two 4-dim centroids each; K <= 256
      // gives at most 8 per lane, all requested before the first is used
      const int n = K * DS / 8;
      const uint4* src = reinterpret_cast<const uint4*>(p.pq_cb) + (size_t)part * n;
      uint4* dst = reinterpret_cast<uint4*>(s_pq) + (size_t)part * n;
      uint4 cl[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (lane + 32 * j < n) cl[j] = __ldg(src + lane + 32 * j);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = lane + 32 * j;
        if (i >= n) break;
        const uint4 c = cl[j];
        dst[i] = c;
        const uint32_t w4[4] = {c.x, c.y, c.z, c.w};
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[k]));
          if (DS == 8 || k < 2) {
            s0 = __fmaf_rn(f.x, f.x, s0);
            s0 = __fmaf_rn(f.y, f.y, s0);
          } else {
            s1 = __fmaf_rn(f.x, f.x, s1);
            s1 = __fmaf_rn(f.y, f.y, s1);
          }
        }
        if (DS == 8) {
          s_pqcc[part * K + i] = s0;
        } else {
          s_pqcc[part * K + 2 * i] = s0;
          s_pqcc[part * K + 2 * i + 1] = s1;
        }
      }
    }
    if (p.L > 0) {
      for (int i = threadIdx.x; i < Kr * 8; i += nthr) {
        const int c = i >> 3, q = i & 7;
        s_rvq[swz(c, q)] = __ldg(reinterpret_cast<const uint4*>(p.rvq_cb) + i);
      }
      __syncthreads();
      for (int i = threadIdx.x; i < Kr; i += nthr) {
        float s = 0.f;
        for (int q = 0; q < 8; ++q) {
          const uint4 r = s_rvq[swz(i, q)];
          const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[k]));
            s = __fmaf_rn(f.x, f.x, s);
            s = __fmaf_rn(f.y, f.y, s);
          }
        }
        s_rcc[i] = s;
      }
    }
  } else {
    for (int i = threadIdx.x; i < M * K * DS / 8; i += nthr)
      reinterpret_cast<uint4*>(s_pq)[i] = __ldg(reinterpret_cast<const uint4*>(p.pq_cb) + i);
    if (p.L > 0) {
      for (int i = threadIdx.x; i < Kr * 8; i += nthr) {
        const int c = i >> 3, q = i & 7;
        s_rvq[swz(c, q)] = __ldg(reinterpret_cast<const uint4*>(p.rvq_cb) + i);
      }
    }
    __syncthreads();  // norms are summed from the staged copies
    for (int i = threadIdx.x; i < M * K; i += nthr) {
      const uint16_t* c = s_pq + (size_t)i * DS;
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < DS; ++k) {
        const float v = h2f(c[k]);
        s = __fmaf_rn(v, v, s);
      }
      s_pqcc[i] = s;
    }
    if (p.L > 0) {
      for (int i = threadIdx.x; i < Kr; i += nthr) {
        float s = 0.f;
        for (int q = 0; q < 8; ++q) {
          const uint4 r = s_rvq[swz(i, q)];
          const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[k]));
            s = __fmaf_rn(f.x, f.x, s);
            s = __fmaf_rn(f.y, f.y, s);
          }
        }
        s_rcc[i] = s;
      }
    }
    __syncthreads();
  }

  // tiles: each group's leader warp (part 0) owns them; in split mode the group's
  // other warps write their subspaces' codes into the leader's s_code
  unsigned char* wb = smem + p.smem_warp + (size_t)(gslot * split) * p.warp_bytes;
  uint4* xt = reinterpret_cast<uint4*>(wb);                    // [16][8 chunks] swizzled x
  uint4* rt = xt + 16 * 8;                                     // [16][8 chunks] swizzled residual
  float* s_xsq = reinterpret_cast<float*>(rt + 16 * 8);        // [16][M]
  float* s_rr = s_xsq + 16 * M;                                // [16]
  uint8_t* s_code = reinterpret_cast<uint8_t*>(s_rr + 16);    // [16][M]
  uint8_t* s_rcode = s_code + 16 * M;                          // [16]
  uint8_t* s_act = s_rcode + 16;                               // [16]

  const int r0 = lane >> 2, qd = lane & 3;
  const float INF = __int_as_float(0x7f800000);

  // the round count is the same for every warp of the CTA (split mode syncs the CTA)
  for (int64_t base = (int64_t)blockIdx.x * gpc; base < ngroups; base += (int64_t)gridDim.x * gpc) {
    const int64_t gg = base + gslot;
    const bool live = gg < ngroups;
    const bool isv = p.x_v != nullptr && gg >= p.ngk;  // a V group of a K+V launch
    const int64_t g = isv ? gg - p.ngk : gg;           // group index within its tensor
    const int kvf = isv ? 1 : p.kv;
    // ---- x tile (leader) ----
    if (live && lead) {
      uint4 xr[4];
      if (split > 1 && base == (int64_t)blockIdx.x * gpc) {
#pragma unroll
        for (int s = 0; s < 4; ++s) xr[s] = xpre[s];
      } else {
        fetch_x(p, gg, lane, xr);
      }
#pragma unroll
      for (int s = 0; s < 4; ++s) xt[swz((lane >> 3) + 4 * s, lane & 7)] = xr[s];
      __syncwarp();
      // |x_m|^2 per (vector, subspace), sequential fp32 (quantization.py:94)
      for (int idx = lane; idx < 16 * M; idx += 32) {
        const int i = idx / M, m = idx - i * M;
        const uint16_t* xr = reinterpret_cast<const uint16_t*>(&xt[swz(i, (m * DS) >> 3)]) + ((m * DS) & 7);
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < DS; ++k) {
          const float v = h2f(xr[k]);
          s = __fmaf_rn(v, v, s);
        }
        s_xsq[idx] = s;
      }
      __syncwarp();
    }
    if (split > 1) __syncthreads();

    // ---- PQ: per-subspace argmin over K centroids (subspaces part, part + split, ...) ----
    if (live) {
      for (int m = part; m < M; m += split) {
        const int chunk = (m * DS) >> 3;
        const uint32_t* x0 = reinterpret_cast<const uint32_t*>(&xt[swz(r0, chunk)]);
        const uint32_t* x1 = reinterpret_cast<const uint32_t*>(&xt[swz(r0 + 8, chunk)]);
        const uint32_t a0 = x0[qd], a1 = x1[qd];
        const float xx0 = s_xsq[r0 * M + m], xx1 = s_xsq[(r0 + 8) * M + m];
        // B lanes that carry this subspace's dims (4-dim subspaces fill half of k)
        const bool bl = DS == 8 || ((qd >> 1) == (m & 1));
        const uint32_t* cbm = reinterpret_cast<const uint32_t*>(s_pq + (size_t)m * K * DS);
        const float* ccm = s_pqcc + m * K;
        float b00 = INF, b01 = INF, b10 = INF, b11 = INF;  // rows r0 / r0+8, column parity 0 / 1
        int i00 = 0, i01 = 0, i10 = 0, i11 = 0;
#pragma unroll 4
        for (int nt = 0; nt < K / 8; ++nt) {
          const int cb = nt * 8 + r0;  // centroid of this lane's B column
          const uint32_t b = bl ? cbm[(cb * DS >> 1) + (DS == 8 ? qd : (qd & 1))] : 0u;
          float c[4] = {0.f, 0.f, 0.f, 0.f};
          mma1688(c, a0, a1, b);
          const int code = nt * 8 + 2 * qd;
          const float2 cc = *reinterpret_cast<const float2*>(ccm + code);
          float d0, d1, d2, d3;
          dist2(d0, d1, c[0], c[1], xx0, cc.x, cc.y);
          dist2(d2, d3, c[2], c[3], xx1, cc.x, cc.y);
          take_min(d0, code, b00, i00);
          take_min(d1, code + 1, b01, i01);
          take_min(d2, code, b10, i10);
          take_min(d3, code + 1, b11, i11);
        }
        merge_min(b00, i00, b01, i01);
        merge_min(b10, i10, b11, i11);
        quad_min(b00, i00);
        quad_min(b10, i10);
        if (qd == 0) {
          s_code[r0 * M + m] = (uint8_t)i00;
          s_code[(r0 + 8) * M + m] = (uint8_t)i10;
        }
      }
    }
    if (split > 1) __syncthreads(); else __syncwarp();
    // ---- the leader finishes the group; every warp meets the same barriers ----
    if (live && lead) {

      // ---- residual r = fp16(x - c): one rounding of the exact difference ----
      for (int idx = lane; idx < 16 * 8; idx += 32) {
        const int i = idx >> 3, q = idx & 7;
        const uint4 xv = xt[swz(i, q)];
        uint4 cv;
        if constexpr (DS == 8) {
          cv = *reinterpret_cast<const uint4*>(s_pq + ((size_t)q * K + s_code[i * M + q]) * 8);
        } else {
          const uint2 lo = *reinterpret_cast<const uint2*>(s_pq + ((size_t)(2 * q) * K + s_code[i * M + 2 * q]) * 4);
          const uint2 hi =
              *reinterpret_cast<const uint2*>(s_pq + ((size_t)(2 * q + 1) * K + s_code[i * M + 2 * q + 1]) * 4);
          cv = make_uint4(lo.x, lo.y, hi.x, hi.y);
        }
        uint4 rv;
        rv.x = hsub2_u32(xv.x, cv.x); rv.y = hsub2_u32(xv.y, cv.y);
        rv.z = hsub2_u32(xv.z, cv.z); rv.w = hsub2_u32(xv.w, cv.w);
        rt[swz(i, q)] = rv;
        const int64_t v = g * 16 + i;
        if (p.residual_out && v < p.nvec)
          reinterpret_cast<uint4*>(p.residual_out + vec_offset(p, (uint32_t)v))[q] = rv;
      }
      __syncwarp();

      // ---- RVQ, one layer (quantization.py:216-250) ----
      if (p.L > 0) {
        if (lane < 16) {  // norm gate, sequential fp32
          float nn = 0.f;
          for (int q = 0; q < 8; ++q) {
            const uint4 rv = rt[swz(lane, q)];
            const uint32_t w4[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[k]));
              nn = __fmaf_rn(f.x, f.x, nn);
              nn = __fmaf_rn(f.y, f.y, nn);
            }
          }
          s_rr[lane] = nn;
          s_act[lane] = __fsqrt_rn(nn) > p.thr ? 1 : 0;
        }
        __syncwarp();
        uint32_t a[4][4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          a[s][0] = reinterpret_cast<const uint32_t*>(&rt[swz(r0, 2 * s)])[qd];
          a[s][1] = reinterpret_cast<const uint32_t*>(&rt[swz(r0 + 8, 2 * s)])[qd];
          a[s][2] = reinterpret_cast<const uint32_t*>(&rt[swz(r0, 2 * s + 1)])[qd];
          a[s][3] = reinterpret_cast<const uint32_t*>(&rt[swz(r0 + 8, 2 * s + 1)])[qd];
        }
        const float rr0 = s_rr[r0], rr1 = s_rr[r0 + 8];
        float b00 = INF, b01 = INF, b10 = INF, b11 = INF;
        int i00 = 0, i01 = 0, i10 = 0, i11 = 0;
#pragma unroll 2
        for (int nt = 0; nt < Kr / 8; ++nt) {
          const int cb = nt * 8 + r0;
          float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const uint32_t bb0 = reinterpret_cast<const uint32_t*>(&s_rvq[swz(cb, 2 * s)])[qd];
            const uint32_t bb1 = reinterpret_cast<const uint32_t*>(&s_rvq[swz(cb, 2 * s + 1)])[qd];
            mma16816(c, a[s], bb0, bb1);
          }
          const int code = nt * 8 + 2 * qd;
          const float2 cc = *reinterpret_cast<const float2*>(s_rcc + code);
          float d0, d1, d2, d3;
          dist2(d0, d1, c[0], c[1], rr0, cc.x, cc.y);
          dist2(d2, d3, c[2], c[3], rr1, cc.x, cc.y);
          take_min(d0, code, b00, i00);
          take_min(d1, code + 1, b01, i01);
          take_min(d2, code, b10, i10);
          take_min(d3, code + 1, b11, i11);
        }
        merge_min(b00, i00, b01, i01);
        merge_min(b10, i10, b11, i11);
        quad_min(b00, i00);
        quad_min(b10, i10);
        if (qd == 0) {
          s_rcode[r0] = s_act[r0] ? (uint8_t)i00 : 0;
          s_rcode[r0 + 8] = s_act[r0 + 8] ? (uint8_t)i10 : 0;
        }
        __syncwarp();
      }

      // ---- sparse top-S of the fp16 decode error, and the code stores: one lane per vector ----
      if (lane < 16) {
        const int i = lane;
        const int64_t v = g * 16 + i;
        if (v < p.nvec) {
          const uint32_t heads = (uint32_t)p.heads, tokens = (uint32_t)p.tokens;
          const uint32_t bt = (uint32_t)v / heads, h = (uint32_t)v - bt * heads;
          const uint32_t b = bt / tokens, t = bt - b * tokens;
          const int64_t row = (int64_t)b * heads + h, tok = p.first + t;
          const int fk = kvf * 5;
          uint8_t* f_pq = p.data + field_byte(p.lay, p.rows, p.cap, p.slot, row, tok, fk + 0);
          for (int m = 0; m < M; ++m) f_pq[m] = s_code[i * M + m];
          if (p.L > 0) {
            p.data[field_byte(p.lay, p.rows, p.cap, p.slot, row, tok, fk + 1)] = s_rcode[i];
            p.data[field_byte(p.lay, p.rows, p.cap, p.slot, row, tok, fk + 2)] = s_act[i];
          }
          if (p.S > 0) {
            uint8_t* f_spi = p.data + field_byte(p.lay, p.rows, p.cap, p.slot, row, tok, fk + 3);
            uint16_t* f_spv =
                reinterpret_cast<uint16_t*>(p.data + field_byte(p.lay, p.rows, p.cap, p.slot, row, tok, fk + 4));
            // err = x - fp16(pq + rvq) in fp32 (quantization.py:310-319 decode, then the error)
            float err[kTcD];
            const bool act = p.L > 0 && s_act[i];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const uint4 xv = xt[swz(i, q)];
              uint4 cv;  // the decode: PQ centroid, plus the RVQ row in fp16 when active
              if constexpr (DS == 8) {
                cv = *reinterpret_cast<const uint4*>(s_pq + ((size_t)q * K + s_code[i * M + q]) * 8);
              } else {
                const uint2 lo =
                    *reinterpret_cast<const uint2*>(s_pq + ((size_t)(2 * q) * K + s_code[i * M + 2 * q]) * 4);
                const uint2 hi =
                    *reinterpret_cast<const uint2*>(s_pq + ((size_t)(2 * q + 1) * K + s_code[i * M + 2 * q + 1]) * 4);
                cv = make_uint4(lo.x, lo.y, hi.x, hi.y);
              }
              if (act) {
                const uint4 rr = s_rvq[swz(s_rcode[i], q)];
                cv.x = hadd2_u32(cv.x, rr.x); cv.y = hadd2_u32(cv.y, rr.y);
                cv.z = hadd2_u32(cv.z, rr.z); cv.w = hadd2_u32(cv.w, rr.w);
              }
              const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
              const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float2 xf = __half22float2(*reinterpret_cast<const __half2*>(&xw[k]));
                const float2 cf = __half22float2(*reinterpret_cast<const __half2*>(&cw[k]));
                err[8 * q + 2 * k] = __fsub_rn(xf.x, cf.x);
                err[8 * q + 2 * k + 1] = __fsub_rn(xf.y, cf.y);
              }
            }
            unsigned long long taken = 0ull;
            for (int s = 0; s < p.S; ++s) {  // largest |err| not yet taken, ties to the lower index
              float bm = -1.f;
              int bi = 0;
#pragma unroll
              for (int d = 0; d < kTcD; ++d) {
                const float mg = ((taken >> d) & 1ull) ? -2.f : fabsf(err[d]);
                if (mg > bm) {
                  bm = mg;
                  bi = d;
                }
              }
              float ev = 0.f;
#pragma unroll
              for (int d = 0; d < kTcD; ++d) ev = d == bi ? err[d] : ev;
              taken |= 1ull << bi;
              f_spi[s] = (uint8_t)bi;
              f_spv[s] = f2h(ev);
            }
          }
        }
      }
    }  // leader
    if (split > 1) __syncthreads(); else __syncwarp();
  }
}

bool encode_tc_supported(const rfsn_quantizer* qz) {
  return qz->head_dim == kTcD && (qz->subspace_dim == 4 || qz->subspace_dim == 8) && qz->pq_codebook_size % 8 == 0 &&
         qz->pq_codebook_size <= 256 && (qz->rvq_layers == 0 || (qz->rvq_layers == 1 && qz->rvq_codebook_size % 8 == 0 &&
                                                                  qz->rvq_codebook_size <= 256)) &&
         qz->sparse_topk <= kTcD;
}

int encode_tc_launch(const rfsn_quantizer* qz, const uint16_t* x, const uint16_t* x_v, int64_t batch,
                     int64_t tokens, int64_t heads, int64_t sb, int64_t st, int64_t sh, const rfsn_code_store* dst,
                     int kv, int64_t slot, int64_t first, uint16_t* residual_out, cudaStream_t stream) {
  if (x_v && (kv != 0 || residual_out)) return RFSN_ERR_INVALID_ARGUMENT;
  EncTcParams p{};
  p.x = x;
  p.x_v = x_v;
  p.batch = batch; p.tokens = tokens; p.heads = heads; p.sb = sb; p.st = st; p.sh = sh;
  p.nvec = batch * tokens * heads;
  p.data = dst->data;
  p.lay = layout_of(qz);
  p.kv = kv;
  p.cap = dst->cap; p.rows = dst->rows; p.slot = slot; p.first = first;
  p.residual_out = residual_out;
  p.pq_cb = qz->pq_codebooks;
  p.rvq_cb = qz->rvq_codebooks;
  p.M = qz->num_subspaces; p.K = qz->pq_codebook_size; p.L = qz->rvq_layers; p.Kr = qz->rvq_codebook_size;
  p.S = qz->sparse_topk;
  p.thr = qz->rvq_threshold;
  int64_t off = 0;
  p.smem_pq = (int)off; off = align_up(off + (int64_t)p.M * p.K * qz->subspace_dim * 2, 128);
  p.smem_pqcc = (int)off; off = align_up(off + (int64_t)p.M * p.K * 4, 128);
  p.smem_rvq = (int)off; off = align_up(off + (int64_t)(p.L ? p.Kr : 0) * kTcD * 2, 128);
  p.smem_rcc = (int)off; off = align_up(off + (int64_t)(p.L ? p.Kr : 0) * 4, 128);
  p.warp_bytes = (int)align_up(2 * 16 * 128 + 16 * p.M * 4 + 16 * 4 + 16 * p.M + 16 + 16, 128);
  p.smem_warp = (int)off; off += (int64_t)kTcWarps * p.warp_bytes;
  if (off > 227 * 1024) return RFSN_ERR_UNSUPPORTED;
  if (p.nvec == 0) return RFSN_OK;
  if (p.nvec >= (int64_t(1) << 31)) return RFSN_ERR_UNSUPPORTED;  // 32-bit vector indexing
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  p.ngk = (p.nvec + 15) / 16;
  const int64_t groups = x_v ? 2 * p.ngk : p.ngk;
  // split mode (one warp per subspace) when its grid fits in one wave of CTAs: a
  // decode step's append is a handful of groups, and a warp walking all M subspaces
  // alone would set the kernel's duration
  const int64_t split_ctas = (groups * p.M + kTcWarps - 1) / kTcWarps;
  p.split = (kTcWarps % p.M == 0 && split_ctas <= sms) ? p.M : 1;
  // split mode runs one group per CTA when that still fits one wave (the search of a
  // subspace is ALU-bound: fewer warps per SM finish it sooner)
  int warps = kTcWarps;
  int64_t want = p.split > 1 ? split_ctas : (groups + kTcWarps - 1) / kTcWarps;
  if (p.split > 1 && groups <= sms) {
    warps = p.split;
    want = groups;
  }
  const int grid = (int)(want < sms ? want : sms);
  cudaError_t e;
  if (qz->subspace_dim == 8) {
    e = cudaFuncSetAttribute(encode_tc_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)off);
    if (e == cudaSuccess) {
      encode_tc_kernel<8><<<grid, warps * 32, off, stream>>>(p);
      e = cudaGetLastError();
    }
  } else {
    e = cudaFuncSetAttribute(encode_tc_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)off);
    if (e == cudaSuccess) {
      encode_tc_kernel<4><<<grid, warps * 32, off, stream>>>(p);
      e = cudaGetLastError();
    }
  }
  return check_cuda(e);
}

}  // namespace rfsn
