// rfsn_attn_chunk.cuh — one warp's work on one 16-token chunk of a tile.
//
// A chunk is 4 row-steps of 4 tokens; lane (slot, j) handles token slot of a
// row-step and dims [j*D/8, (j+1)*D/8).  Work is written as straight-line
// phases over pairs of row-steps (all code loads, then all codebook gathers,
// then arithmetic) so shared-memory latency overlaps across tokens; tokens
// past the tile end read token 0's data (always valid) and are masked out of
// the softmax instead of branched around.
//
// Modes: kDense (hot fp16 rows), kRvq1 (PQ + one uint8 RVQ layer staged in
// shared memory, sparse S <= 8), kPqOnly (PQ, sparse S <= 8), kGeneric (any
// RVQ layout / sparse width, via recon_lane).  PQ codebooks are staged
// code-major ([K][M][ds]) so one token's 8 lanes read 8 distinct banks; with
// 4-dim subspaces odd token slots load their two centroids in swapped order
// so a half-warp (two tokens) stays conflict-free.
#pragma once

#include "rfsn_attn_util.cuh"
#include "rfsn_common.cuh"
#include "rfsn_layout.h"

namespace rfsn {

enum ChunkMode { kDense = 0, kRvq1 = 1, kPqOnly = 2, kGeneric = 3 };

struct TileView {
  const unsigned char* base;  // compressed tiles: the stage holding whole 16-token blocks
  int t0;                     // index of the tile's first token inside the first block
  int kvo;                    // field offset: 0 = K fields, 5 = V fields
  const uint16_t* dense;      // hot fp16 rows (dense tiles)
};

struct ChunkShared {
  const uint16_t* pq_cm;    // code-major PQ codebook [K][M][ds] (shared)
  const uint16_t* rvq_s;    // RVQ codebook [L][Kr][D] (shared, when staged)
  const uint16_t* rvq_g;    // RVQ codebook in global memory
  const float* qtab;        // this warp's fp32 query table [D][RMAX]
  float* vsp;               // this warp's sparse-V sums [4][D][RMAX]
  int M, K, ds, L, Kr, S, rvq_u16, rvq_smem, has_mask, rvq_bpt;
  BlockLayout lay;          // field offsets inside a 16-token block
  int n, pos0, R, causal, qp_lane;
  float sl2;                // scale * log2(e)
};

// code-major PQ gather of one lane's 8 dims [d0, d0+8) (fast paths).
template <int DS>
__device__ __forceinline__ void pq8_cm(const uint16_t* cm, int M, const unsigned char* codes, int d0, bool odd,
                                       uint32_t* o) {
  if constexpr (DS == 4) {
    const int m0 = d0 >> 2;
    const uint32_t c01 = *reinterpret_cast<const uint16_t*>(codes + m0);
    const uint32_t c0 = c01 & 0xffu, c1 = c01 >> 8;
    // odd slots read subspace m0+1 first: the two tokens of a half-warp hit
    // complementary bank halves
    const uint32_t ma = odd ? m0 + 1 : m0, ca = odd ? c1 : c0;
    const uint32_t mb = odd ? m0 : m0 + 1, cb = odd ? c0 : c1;
    const uint2 a = *reinterpret_cast<const uint2*>(cm + ((ca * M + ma) << 2));
    const uint2 b = *reinterpret_cast<const uint2*>(cm + ((cb * M + mb) << 2));
    o[0] = odd ? b.x : a.x;
    o[1] = odd ? b.y : a.y;
    o[2] = odd ? a.x : b.x;
    o[3] = odd ? a.y : b.y;
  } else {  // DS == 8
    const int m = d0 >> 3;
    const uint4 a = *reinterpret_cast<const uint4*>(cm + (((uint32_t)codes[m] * M + m) << 3));
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
  }
}

// generic code-major PQ gather (any ds)
__device__ __forceinline__ void pq8_cm_generic(const uint16_t* cm, int M, int ds, const unsigned char* codes, int d0,
                                               uint32_t* o) {
  if (ds >= 8) {
    const int m = d0 / ds, off = d0 - m * ds;
    const uint4 a = *reinterpret_cast<const uint4*>(cm + ((uint32_t)codes[m] * M + m) * ds + off);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
  } else if (ds == 4) {
    const int m = d0 >> 2;
    const uint2 a = *reinterpret_cast<const uint2*>(cm + (((uint32_t)codes[m] * M + m) << 2));
    const uint2 b = *reinterpret_cast<const uint2*>(cm + (((uint32_t)codes[m + 1] * M + m + 1) << 2));
    o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
  } else if (ds == 2) {
    const int m = d0 >> 1;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = *reinterpret_cast<const uint32_t*>(cm + (((uint32_t)codes[m + i] * M + m + i) << 1));
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = cm[(uint32_t)codes[d0 + 2 * i] * M + d0 + 2 * i];
      const uint32_t hi = cm[(uint32_t)codes[d0 + 2 * i + 1] * M + d0 + 2 * i + 1];
      o[i] = lo | (hi << 16);
    }
  }
}

// Start of field k (0 pq, 1 rvq, 2 active, 3 sp_idx, 4 sp_val) of token t of a tile.
__device__ __forceinline__ const unsigned char* tok_field(const ChunkShared& cs, const TileView& tv, int t, int k) {
  const int ti = tv.t0 + t;
  return tv.base + (ti >> 4) * cs.lay.block_bytes + cs.lay.off[tv.kvo + k] + (ti & 15) * cs.lay.bpt[k];
}

// Reconstruct one lane's dims of token t (tile-local, already clamped to a valid token).
template <int D, int DS, int MODE>
__device__ __forceinline__ void recon_token(const ChunkShared& cs, const TileView& tv, int t, int dim0, bool odd,
                                            uint32_t* w) {
  constexpr int DPL = D / 8;
  if constexpr (MODE == kDense) {
    load_dense<DPL>(tv.dense + (size_t)t * D + dim0, w);
  } else if constexpr (MODE == kRvq1 || MODE == kPqOnly) {
    const unsigned char* codes = tok_field(cs, tv, t, 0);
#pragma unroll
    for (int g8 = 0; g8 < DPL / 8; ++g8) pq8_cm<DS>(cs.pq_cm, cs.M, codes, dim0 + 8 * g8, odd, w + 4 * g8);
    if constexpr (MODE == kRvq1) {
      const bool act = !cs.has_mask || *tok_field(cs, tv, t, 2) != 0;
      const uint32_t c = act ? *tok_field(cs, tv, t, 1) : 0u;
#pragma unroll
      for (int g8 = 0; g8 < DPL / 8; ++g8) {
        const uint4 r = *reinterpret_cast<const uint4*>(cs.rvq_s + c * D + dim0 + 8 * g8);
        w[4 * g8 + 0] = hadd2_u32(w[4 * g8 + 0], act ? r.x : 0u);
        w[4 * g8 + 1] = hadd2_u32(w[4 * g8 + 1], act ? r.y : 0u);
        w[4 * g8 + 2] = hadd2_u32(w[4 * g8 + 2], act ? r.z : 0u);
        w[4 * g8 + 3] = hadd2_u32(w[4 * g8 + 3], act ? r.w : 0u);
      }
    }
  } else {
    const unsigned char* codes = tok_field(cs, tv, t, 0);
#pragma unroll
    for (int g8 = 0; g8 < DPL / 8; ++g8) pq8_cm_generic(cs.pq_cm, cs.M, cs.ds, codes, dim0 + 8 * g8, w + 4 * g8);
    const bool act = cs.L > 0 && (!cs.has_mask || *tok_field(cs, tv, t, 2) != 0);
    if (act) {
      const unsigned char* rc = tok_field(cs, tv, t, 1);
      if (cs.rvq_smem) {
#pragma unroll
        for (int g8 = 0; g8 < DPL / 8; ++g8) rvq_add8<D>(cs.rvq_s, cs.L, cs.Kr, cs.rvq_u16, rc, dim0 + 8 * g8, w + 4 * g8);
      } else {
#pragma unroll
        for (int g8 = 0; g8 < DPL / 8; ++g8) rvq_add8<D>(cs.rvq_g, cs.L, cs.Kr, cs.rvq_u16, rc, dim0 + 8 * g8, w + 4 * g8);
      }
    }
  }
}

// Sparse residual terms handled by this lane for token t: returns sum_e q_r[idx_e] * val_e
// (K side) over entries e = j, j+8, ... < S.
template <int RMAX, int MODE>
__device__ __forceinline__ void sparse_k(const ChunkShared& cs, const TileView& tv, int t, int j, float* corr) {
#pragma unroll
  for (int r = 0; r < RMAX; ++r) corr[r] = 0.f;
  const unsigned char* spi = tok_field(cs, tv, t, 3);
  const uint16_t* spv = reinterpret_cast<const uint16_t*>(tok_field(cs, tv, t, 4));
  if constexpr (MODE == kRvq1 || MODE == kPqOnly) {  // S <= 8: at most one entry per lane
    const bool has = j < cs.S;
    const int e = has ? j : 0;
    const int idx = spi[e];
    const float val = has ? h2f(spv[e]) : 0.f;
    float qv[RMAX];
    load_row<RMAX>(cs.qtab + idx * RMAX, qv);
#pragma unroll
    for (int r = 0; r < RMAX; ++r) corr[r] = qv[r] * val;
  } else {
    for (int e = j; e < cs.S; e += 8) {
      const int idx = spi[e];
      const float val = h2f(spv[e]);
      float qv[RMAX];
      load_row<RMAX>(cs.qtab + idx * RMAX, qv);
#pragma unroll
      for (int r = 0; r < RMAX; ++r) corr[r] = __fmaf_rn(qv[r], val, corr[r]);
    }
  }
}

// V side: add p_r * val_e into this slot's sparse-V sums for entries of token t.
template <int RMAX, int MODE>
__device__ __forceinline__ void sparse_v(const ChunkShared& cs, const TileView& tv, int t, int j, int slot,
                                         int D, const float* pv) {
  const unsigned char* spi = tok_field(cs, tv, t, 3);
  const uint16_t* spv = reinterpret_cast<const uint16_t*>(tok_field(cs, tv, t, 4));
  if constexpr (MODE == kRvq1 || MODE == kPqOnly) {
    const bool has = j < cs.S;
    const int e = has ? j : 0;
    const int idx = spi[e];
    const float val = has ? h2f(spv[e]) : 0.f;
    float* dst = cs.vsp + ((size_t)slot * D + idx) * RMAX;
    float cur[RMAX];
    load_row<RMAX>(dst, cur);
#pragma unroll
    for (int r = 0; r < RMAX; ++r) cur[r] = __fmaf_rn(pv[r], val, cur[r]);
    store_row<RMAX>(dst, cur);
  } else {
    for (int e = j; e < cs.S; e += 8) {
      const int idx = spi[e];
      const float val = h2f(spv[e]);
      float* dst = cs.vsp + ((size_t)slot * D + idx) * RMAX;
      float cur[RMAX];
      load_row<RMAX>(dst, cur);
#pragma unroll
      for (int r = 0; r < RMAX; ++r) cur[r] = __fmaf_rn(pv[r], val, cur[r]);
      store_row<RMAX>(dst, cur);
    }
  }
}

// One 16-token chunk: scores on tensor cores, online softmax, V accumulation.
template <int D, int RMAX, int DS, int MODE>
__device__ __forceinline__ void process_chunk(const ChunkShared& cs, const TileView& tk, const TileView& tvv,
                                              int cbase, const uint32_t (*aq)[4], const uint32_t (*asp)[4],
                                              float (*acc)[D / 8], float& m_run, float& l_run) {
  constexpr int DPL = D / 8;
  constexpr int NMMA = DPL / 4;
  constexpr int NSP = (RMAX + 3) / 4;
  const float NEG_INF = __int_as_float(0xff800000);
  const int lane = threadIdx.x & 31;
  const int slot = lane >> 3, j = lane & 7, dim0 = j * DPL;
  const int srow = lane >> 2, sslot = lane & 3;
  const bool odd = slot & 1;
  const bool sparse = MODE != kDense && cs.S > 0;

  // ---------------- scores ----------------
  float sc[4];
#pragma unroll
  for (int hs = 0; hs < 2; ++hs) {
    int tc[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int tl = cbase + 4 * (2 * hs + u) + slot;
      tc[u] = tl < cs.n ? tl : 0;
    }
    uint32_t w[2][DPL / 2];
#pragma unroll
    for (int u = 0; u < 2; ++u) recon_token<D, DS, MODE>(cs, tk, tc[u], dim0, odd, w[u]);
    float cfr[2][4];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      cfr[u][0] = cfr[u][1] = cfr[u][2] = cfr[u][3] = 0.f;
#pragma unroll
      for (int s = 0; s < NMMA; ++s) mma16816(cfr[u], aq[s], w[u][2 * s], w[u][2 * s + 1]);
    }
    if (sparse) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float corr[RMAX];
        sparse_k<RMAX, MODE>(cs, tk, tc[u], j, corr);
#pragma unroll
        for (int t = 0; t < NSP; ++t) {
          float c4[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) c4[i] = (4 * t + i < RMAX) ? corr[4 * t + i] : 0.f;
          uint32_t hi01, hi23, lo01, lo23;
          split_h2(c4[0], c4[1], hi01, lo01);
          split_h2(c4[2], c4[3], hi23, lo23);
          mma16816(cfr[u], asp[t], hi01, hi23);
          mma16816(cfr[u], asp[t], lo01, lo23);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int stl = cbase + 4 * (2 * hs + u) + sslot;
      const bool allowed = stl < cs.n && srow < cs.R && (!cs.causal || cs.pos0 + stl <= cs.qp_lane);
      sc[2 * hs + u] = allowed ? (cfr[u][0] + cfr[u][3]) * cs.sl2 : NEG_INF;
    }
  }

  // ---------------- online softmax of row srow over the 16 tokens ----------------
  float cmax = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
  cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 1));
  cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 2));
  const float m_new = fmaxf(m_run, cmax);
  float alpha = 1.f;
  if (m_new > m_run) alpha = (m_run == NEG_INF) ? 0.f : ex2_approx(m_run - m_new);
  float pr[4];
  float lsum = 0.f;
#pragma unroll
  for (int rs = 0; rs < 4; ++rs) {
    pr[rs] = (sc[rs] == NEG_INF) ? 0.f : ex2_approx(sc[rs] - m_new);
    lsum += pr[rs];
  }
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
  l_run = l_run * alpha + lsum;
  m_run = m_new;
  if (__any_sync(0xffffffffu, alpha != 1.f)) {  // a row's max grew: rescale its sums
    float arow[RMAX];
#pragma unroll
    for (int r = 0; r < RMAX; ++r) arow[r] = __shfl_sync(0xffffffffu, alpha, 4 * r);
#pragma unroll
    for (int r = 0; r < RMAX; ++r)
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[r][i] *= arow[r];
    if (cs.S > 0) {
#pragma unroll
      for (int r = 0; r < RMAX; ++r)
        for (int k = lane; k < 4 * D; k += 32) cs.vsp[k * RMAX + r] *= arow[r];
    }
    __syncwarp();
  }

  // ---------------- values ----------------
#pragma unroll
  for (int hs = 0; hs < 2; ++hs) {
    int tc[2];
    float pv[2][RMAX];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int tl = cbase + 4 * (2 * hs + u) + slot;
      tc[u] = tl < cs.n ? tl : 0;
#pragma unroll
      for (int r = 0; r < RMAX; ++r) pv[u][r] = __shfl_sync(0xffffffffu, pr[2 * hs + u], 4 * r + slot);
    }
    uint32_t w[2][DPL / 2];
#pragma unroll
    for (int u = 0; u < 2; ++u) recon_token<D, DS, MODE>(cs, tvv, tc[u], dim0, odd, w[u]);
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int i = 0; i < DPL / 2; ++i) {
        const float2 v2 = __half22float2(*reinterpret_cast<const __half2*>(&w[u][i]));
#pragma unroll
        for (int r = 0; r < RMAX; ++r) ffma2(acc[r][2 * i], acc[r][2 * i + 1], pv[u][r], v2.x, v2.y);
      }
    if (sparse) {
#pragma unroll
      for (int u = 0; u < 2; ++u) sparse_v<RMAX, MODE>(cs, tvv, tc[u], j, slot, D, pv[u]);
    }
  }
}

}  // namespace rfsn
