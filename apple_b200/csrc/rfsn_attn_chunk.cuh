// rfsn_attn_chunk.cuh — one consumer warp's work on one 16-token block of a tile.
//
// A chunk is one 16-token block of the code store (or 16 hot rows): 4
// row-steps of 4 tokens; lane (slot, j) handles token 4*rs + slot of the block
// and dims [j*D/8, (j+1)*D/8).  Work is straight-line phases over pairs of
// row-steps so shared-memory latency overlaps across tokens; tokens outside
// the tile's valid range [t_lo, t_hi) are masked in the softmax instead of
// branched around.
//
// Exact values.  A lane rebuilds its dims the way the reference decodes them
// (quantization.py:310-319): fp16 PQ centroid + fp16 RVQ row (one layer) or
// fp16(fp32 sum of rows), fp16 add.  The top-S sparse residual is applied as
// materialisation does, value = fp16(recon + val): each lane writes its
// token's entries into a per-warp fp16 scratch row [slot][D] (a token's
// entries have distinct dims), the warp syncs, and every lane reads back its
// own dims as 16-byte loads, adds them with __hadd2 and zeroes them.  Two
// sets of scatter rows alternate between consecutive rounds, so the __syncwarp
// of one round orders the previous round's zeroing before the next writes to
// the same set.  fp32 addition of two fp16 values followed by one rounding to
// fp16 equals the correctly rounded fp16 sum (24 >= 2*11+1 bits), so __hadd2
// reproduces the fp32-then-round decode exactly.
//
// Layout presets (LP) fix the block layout at compile time for the common
// D = 64 configurations, so field addresses are block base + immediates.  The
// PQ codebook is staged code-major ([K][M][ds]); with 4-dim subspaces odd
// token slots read a second copy whose subspace pairs are swapped, so the two
// tokens of a half-warp cover all 32 banks once with no selects.
#pragma once

#include "rfsn_attn_util.cuh"
#include "rfsn_common.cuh"
#include "rfsn_layout.h"

namespace rfsn {

enum LayoutPreset {
  kGeneric = 0,         // runtime layout: any ds, RVQ depth, code width, sparse width, D = 64 or 128
  kDs4Rvq1DenseS8 = 1,  // D=64, PQ 16x4 K=256, one uint8 RVQ layer (Kr=256) on every token, top-8 sparse
  kDs4Rvq1Mask = 2,     // D=64, PQ 16x4 K=256, one uint8 RVQ layer gated by activity bytes, no sparse
  kDs8PqOnly = 3,       // D=64, PQ 8x8 K=256, no RVQ, no sparse
  kDs8Rvq1Mask = 4,     // D=64, PQ 8x8 K=256, one uint8 RVQ layer gated by activity bytes, no sparse
};

template <int LP>
struct Preset {
  static constexpr int DS = (LP == kDs4Rvq1DenseS8 || LP == kDs4Rvq1Mask) ? 4 : 8;
  static constexpr int M = 64 / DS;
  static constexpr int L = (LP == kDs8PqOnly) ? 0 : 1;
  static constexpr bool MASK = (LP == kDs4Rvq1Mask || LP == kDs8Rvq1Mask);
  static constexpr int S = (LP == kDs4Rvq1DenseS8) ? 8 : 0;
  // field offsets inside a block: K fields, then the same V fields at FB
  static constexpr int OPQ = 0;
  static constexpr int ORVQ = OPQ + 16 * M;
  static constexpr int OACT = ORVQ + 16 * L;
  static constexpr int OSPI = OACT + 16 * L;
  static constexpr int OSPV = OSPI + 16 * S;
  static constexpr int FB = OSPV + 32 * S;
  static constexpr int BLOCK = 2 * FB;
};

// True when the runtime block layout equals preset LP's compile-time one.
template <int LP>
__host__ inline bool preset_layout_matches(const BlockLayout& b) {
  using P = Preset<LP>;
  const int want[5] = {P::OPQ, P::ORVQ, P::OACT, P::OSPI, P::OSPV};
  const int bpt[5] = {P::M, P::L, P::L, P::S, 2 * P::S};
  for (int k = 0; k < 5; ++k) {
    if (b.bpt[k] != bpt[k]) return false;
    if (bpt[k] && (b.off[k] != want[k] || b.off[5 + k] != P::FB + want[k])) return false;
  }
  return b.block_bytes == P::BLOCK;
}

struct ChunkCtx {
  const uint16_t* pq_cm;   // code-major PQ codebook [K][M][ds] (shared)
  const uint16_t* pq_sel;  // this lane's copy: pq_cm, or the pair-swapped copy for odd slots (4-dim presets)
  const uint16_t* pq_vsel; // PQ-only preset: this lane's copy for V gathers (subspace m at m ^ 2(lane%4))
  const uint16_t* rvq_s;   // RVQ codebook [L][Kr][D] (shared, when staged)
  const uint16_t* rvq_g;   // RVQ codebook (global)
  uint16_t* scratch;       // this warp's sparse scatter rows [2 sets][tokens per round][4 slots][D] fp16
  BlockLayout lay;         // runtime block layout (generic path)
  int M, K, ds, L, Kr, S, rvq_u16, rvq_smem, has_mask;
  int qp_lim;              // score lane's row: last visible position (causal), huge (not causal), very negative (unused row)
  float sl2;               // softmax scale * log2(e)
};

// Fast path: this lane's 8 dims of token tb of a block, K (kv = 0) or V (kv = 1) fields.
// rvq_in / act_in: the token's RVQ code and activity byte when the caller has them
// already (one 16-byte load per field and phase), else -1 to read them here.
template <int LP>
__device__ __forceinline__ void recon_fast(const ChunkCtx& c, const unsigned char* blk, int kv, int tb, int j,
                                           bool odd, uint32_t* w, int rvq_in = -1, int act_in = -1) {
  using P = Preset<LP>;
  const unsigned char* f = blk + kv * P::FB;
  if constexpr (P::DS == 4) {
    const int m0 = 2 * j;
    const uint32_t c01 = *reinterpret_cast<const uint16_t*>(f + P::OPQ + tb * P::M + m0);
    const uint32_t c0 = c01 & 0xffu, c1 = c01 >> 8;
    // odd slots: the swapped copy holds subspace m0 at position m0+1 and vice versa
    const int pa = odd ? 1 : 0;
    const uint2 a = *reinterpret_cast<const uint2*>(c.pq_sel + ((c0 * P::M + m0 + pa) << 2));
    const uint2 b = *reinterpret_cast<const uint2*>(c.pq_sel + ((c1 * P::M + m0 + 1 - pa) << 2));
    w[0] = a.x; w[1] = a.y; w[2] = b.x; w[3] = b.y;
  } else {
    const uint32_t cc = f[P::OPQ + tb * P::M + j];
    const uint4 a = *reinterpret_cast<const uint4*>(c.pq_cm + ((cc * P::M + j) << 3));
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  }
  if constexpr (P::L == 1) {
    const uint32_t code = rvq_in >= 0 ? (uint32_t)rvq_in : f[P::ORVQ + tb];
    if constexpr (P::MASK) {
      const bool act = (act_in >= 0 ? act_in : f[P::OACT + tb]) != 0;
      const uint4 r = *reinterpret_cast<const uint4*>(c.rvq_s + (act ? code : 0u) * 64 + 8 * j);
      w[0] = hadd2_u32(w[0], act ? r.x : 0u); w[1] = hadd2_u32(w[1], act ? r.y : 0u);
      w[2] = hadd2_u32(w[2], act ? r.z : 0u); w[3] = hadd2_u32(w[3], act ? r.w : 0u);
    } else {
      const uint4 r = *reinterpret_cast<const uint4*>(c.rvq_s + code * 64 + 8 * j);
      w[0] = hadd2_u32(w[0], r.x); w[1] = hadd2_u32(w[1], r.y);
      w[2] = hadd2_u32(w[2], r.z); w[3] = hadd2_u32(w[3], r.w);
    }
  }
}

// Generic path: runtime layout.  Codes are clamped to the codebook sizes so a
// store holding stray bytes (tokens outside the window) never indexes past them.
template <int D>
__device__ __forceinline__ void recon_generic(const ChunkCtx& c, const unsigned char* blk, int kv, int tb, int dim0,
                                              uint32_t* w) {
  constexpr int DPL = D / 8;
  const unsigned char* codes = blk + c.lay.off[kv * 5 + 0] + tb * c.lay.bpt[0];
  const uint32_t kmax = (uint32_t)c.K - 1u;
#pragma unroll
  for (int g8 = 0; g8 < DPL / 8; ++g8) {
    const int d0 = dim0 + 8 * g8;
    uint32_t* o = w + 4 * g8;
    if (c.ds >= 8) {
      const int m = d0 / c.ds, off = d0 - m * c.ds;
      const uint32_t cc = min((uint32_t)codes[m], kmax);
      const uint4 a = *reinterpret_cast<const uint4*>(c.pq_cm + (cc * c.M + m) * c.ds + off);
      o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    } else if (c.ds == 4) {
      const int m = d0 >> 2;
      const uint32_t ca = min((uint32_t)codes[m], kmax), cb = min((uint32_t)codes[m + 1], kmax);
      const uint2 a = *reinterpret_cast<const uint2*>(c.pq_cm + ((ca * c.M + m) << 2));
      const uint2 b = *reinterpret_cast<const uint2*>(c.pq_cm + ((cb * c.M + m + 1) << 2));
      o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
    } else if (c.ds == 2) {
      const int m = d0 >> 1;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t cc = min((uint32_t)codes[m + i], kmax);
        o[i] = *reinterpret_cast<const uint32_t*>(c.pq_cm + ((cc * c.M + m + i) << 1));
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t ca = min((uint32_t)codes[d0 + 2 * i], kmax), cb = min((uint32_t)codes[d0 + 2 * i + 1], kmax);
        const uint32_t lo = c.pq_cm[ca * c.M + d0 + 2 * i];
        const uint32_t hi = c.pq_cm[cb * c.M + d0 + 2 * i + 1];
        o[i] = lo | (hi << 16);
      }
    }
  }
  const bool act = c.L > 0 && (!c.has_mask || blk[c.lay.off[kv * 5 + 2] + tb] != 0);
  if (act) {
    const unsigned char* rc = blk + c.lay.off[kv * 5 + 1] + tb * c.lay.bpt[1];
    const uint16_t* cb = c.rvq_smem ? c.rvq_s : c.rvq_g;
#pragma unroll
    for (int g8 = 0; g8 < DPL / 8; ++g8) rvq_add8<D>(cb, c.L, c.Kr, c.rvq_u16, rc, dim0 + 8 * g8, w + 4 * g8);
  }
}

// Sparse residual of TPR tokens of this lane (token tb[i] = row-step rs0+i):
// scatter every entry into this round's fp16 rows, sync the warp, then add
// this lane's dims and zero them.  Rows of a round: [TPR][4 slots][D]; two
// row sets alternate by round parity (the sync of a round orders the previous
// round's zeroing before this round's writes into the same set).
template <int D, int LP, int TPR>
__device__ __forceinline__ void sparse_round(const ChunkCtx& c, const unsigned char* blk, int kv, const int* tb,
                                             const bool* valid, int round, int slot, int j, int dim0,
                                             uint32_t (*w)[D / 16]) {
  constexpr int DPL = D / 8;
  uint16_t* set = c.scratch + (round & 1) * (TPR * 4 * D);
#pragma unroll
  for (int i = 0; i < TPR; ++i) {
    uint16_t* row = set + (i * 4 + slot) * D;
    if constexpr (LP != kGeneric) {
      using P = Preset<LP>;
      const unsigned char* f = blk + kv * P::FB;
      const int idx = f[P::OSPI + tb[i] * P::S + j] & (D - 1);
      const uint16_t val = *reinterpret_cast<const uint16_t*>(f + P::OSPV + (tb[i] * P::S + j) * 2);
      row[idx] = valid[i] ? val : (uint16_t)0;
    } else {
      const unsigned char* spi = blk + c.lay.off[kv * 5 + 3] + tb[i] * c.S;
      const uint16_t* spv = reinterpret_cast<const uint16_t*>(blk + c.lay.off[kv * 5 + 4]) + tb[i] * c.S;
      for (int e = j; e < c.S; e += 8) row[spi[e] & (D - 1)] = valid[i] ? spv[e] : (uint16_t)0;
    }
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < TPR; ++i) {
    uint16_t* src = set + (i * 4 + slot) * D + dim0;
#pragma unroll
    for (int g8 = 0; g8 < DPL / 8; ++g8) {
      uint4* p4 = reinterpret_cast<uint4*>(src + 8 * g8);
      const uint4 d = *p4;
      w[i][4 * g8 + 0] = hadd2_u32(w[i][4 * g8 + 0], d.x);
      w[i][4 * g8 + 1] = hadd2_u32(w[i][4 * g8 + 1], d.y);
      w[i][4 * g8 + 2] = hadd2_u32(w[i][4 * g8 + 2], d.z);
      w[i][4 * g8 + 3] = hadd2_u32(w[i][4 * g8 + 3], d.w);
      *p4 = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// Rebuild this lane's dims of its TPR tokens tb[i] (K or V fields), all loads
// of the round issued before any is used.
// NB: 16-token blocks per chunk; token tb of the chunk lives in block tb / 16
// (consecutive blocks of a tile are adjacent in shared memory).
// rq / ra (fixed layouts with one RVQ layer, one-block chunks): the phase's 16 RVQ
// codes / activity bytes as 4 words; token 4 rs + slot of round-token rs = rsbase + i is
// byte `slot` of word rs.
template <int D, int LP, bool DENSE, int TPR, int NB = 1>
__device__ __forceinline__ void load_round(const ChunkCtx& c, const unsigned char* blk, const uint16_t* dense,
                                           int kv, const int* tb, const bool* valid, int t_lo, int round, int slot,
                                           int j, int dim0, bool odd, uint32_t (*w)[D / 16],
                                           const uint32_t* rq = nullptr, const uint32_t* ra = nullptr,
                                           int rsbase = 0) {
  constexpr int DPL = D / 8;
  static_assert(NB == 1 || (LP != kGeneric && Preset<LP>::S == 0), "multi-block chunks: fixed layouts without sparse");
#pragma unroll
  for (int i = 0; i < TPR; ++i) {
    if constexpr (DENSE) {
      load_dense<DPL>(dense + (valid[i] ? tb[i] : t_lo) * D + dim0, w[i]);
    } else if constexpr (LP != kGeneric && NB > 1) {
      recon_fast<LP>(c, blk + (tb[i] >> 4) * Preset<LP>::BLOCK, kv, tb[i] & 15, j, odd, w[i]);
    } else if constexpr (LP != kGeneric && Preset<LP>::L == 1) {
      const int code = (int)((rq[rsbase + i] >> (8 * slot)) & 0xffu);
      const int act = Preset<LP>::MASK ? (int)((ra[rsbase + i] >> (8 * slot)) & 0xffu) : -1;
      recon_fast<LP>(c, blk, kv, tb[i], j, odd, w[i], code, act);
    } else if constexpr (LP != kGeneric) {
      recon_fast<LP>(c, blk, kv, tb[i], j, odd, w[i]);
    } else {
      recon_generic<D>(c, blk, kv, tb[i], dim0, w[i]);
    }
  }
  if constexpr (!DENSE && (LP == kGeneric || Preset<LP>::S > 0)) {
    if (c.S > 0) sparse_round<D, LP, TPR>(c, blk, kv, tb, valid, round, slot, j, dim0, w);
  }
}

// One chunk of NB 16-token blocks: K scores on tensor cores, online softmax,
// then P.V on tensor cores.  blk: the first block's bytes (code tiles; the next
// block follows it); dense_k/dense_v: the chunk's hot rows (dense tiles).  Valid
// tokens are [t_lo, t_hi); token tb is at position pos_base + tb.  TPR tokens per lane are loaded per round (4 / TPR
// rounds per phase); a round's loads are all in flight before its arithmetic.
//
// Output accumulators (D/16 tiles x 4 per lane): lane (g = lane/4, q = lane%4)
// holds acc[u] = {O[2q][DPL*g+2u], O[2q+1][DPL*g+2u], O[2q][DPL*g+2u+1],
// O[2q+1][DPL*g+2u+1]} for query rows 2q, 2q+1 (unnormalised, online-softmax
// scaled) -- the D fragment of O^T = V^T P^T.
//
// FULL: every token of the block is valid and visible to every live query row
// (the common case; the caller decides it warp-uniformly), so the per-token
// range checks and score masks compile away.  Rows past the KV head's query
// count then score 0 instead of being masked; their state is never read.
template <int D, int RMAX, int LP, bool DENSE, int TPR, bool FULL, int NB = 1>
__device__ __forceinline__ void process_block(const ChunkCtx& c, const unsigned char* blk, const uint16_t* dense_k,
                                              const uint16_t* dense_v, int t_lo, int t_hi, int pos_base,
                                              const uint32_t (*aq)[4], float (*acc)[4], float& m_run,
                                              float& l_run) {
  constexpr int DPL = D / 8;
  constexpr int NT = D / 16;        // P.V tiles of 16 dims
  constexpr int NMMA = DPL / 4;
  constexpr int NR = 4 * NB / TPR;  // rounds per phase
  constexpr int NS = 4 * NB;        // scores per lane (tokens 4 rs + lane%4)
  static_assert(TPR == 2 || TPR == 4, "P.V takes the tokens of a round as one k8 (2) or k16 (4) step");
  static_assert(RMAX <= 8, "P.V covers at most 8 query rows");
  const float NEG_INF = __int_as_float(0xff800000);
  const int lane = threadIdx.x & 31;
  const int slot = lane >> 3, j = lane & 7, dim0 = j * DPL;
  const int sslot = lane & 3;
  const bool odd = slot & 1;
  // score lane (row lane/4, token slot sslot): visible tokens are [t_lo, s_hi)
  const int s_hi = min(t_hi, c.qp_lim - pos_base + 1);

  // one broadcast 16-byte load per field and phase for the RVQ codes / activity bytes
  constexpr bool kCodeWords = !DENSE && LP != kGeneric && NB == 1 && Preset<LP>::L == 1;
  uint32_t rq[4] = {0u, 0u, 0u, 0u}, ra[4] = {0u, 0u, 0u, 0u};
  if constexpr (kCodeWords) {
    using P = Preset<LP>;
    const uint4 r4 = *reinterpret_cast<const uint4*>(blk + P::ORVQ);
    rq[0] = r4.x; rq[1] = r4.y; rq[2] = r4.z; rq[3] = r4.w;
    if constexpr (P::MASK) {
      const uint4 a4 = *reinterpret_cast<const uint4*>(blk + P::OACT);
      ra[0] = a4.x; ra[1] = a4.y; ra[2] = a4.z; ra[3] = a4.w;
    }
  }

  // ---------------- scores ----------------
  float sc[NS];
#pragma unroll
  for (int rr = 0; rr < NR; ++rr) {
    int tb[TPR];
    bool valid[TPR];
#pragma unroll
    for (int i = 0; i < TPR; ++i) {
      tb[i] = 4 * (rr * TPR + i) + slot;
      valid[i] = FULL || (tb[i] >= t_lo && tb[i] < t_hi);
    }
    uint32_t w[TPR][DPL / 2];
    load_round<D, LP, DENSE, TPR, NB>(c, blk, dense_k, 0, tb, valid, t_lo, rr, slot, j, dim0, odd, w, rq, ra,
                                      rr * TPR);
    float cfr[TPR][4];
#pragma unroll
    for (int i = 0; i < TPR; ++i) {
      cfr[i][0] = cfr[i][1] = cfr[i][2] = cfr[i][3] = 0.f;
#pragma unroll
      for (int s = 0; s < NMMA; ++s) mma16816(cfr[i], aq[s], w[i][2 * s], w[i][2 * s + 1]);
    }
#pragma unroll
    for (int i = 0; i < TPR; ++i) {
      const int stb = 4 * (rr * TPR + i) + sslot;
      const float v = (cfr[i][0] + cfr[i][3]) * c.sl2;
      sc[rr * TPR + i] = (FULL || (stb >= t_lo && stb < s_hi)) ? v : NEG_INF;
    }
  }

  // ---------------- online softmax of row lane/4 over the chunk's tokens ----------------
  float cmax = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
#pragma unroll
  for (int rs = 4; rs < NS; rs += 2) cmax = fmaxf(cmax, fmaxf(sc[rs], sc[rs + 1]));
  cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 1));
  cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 2));
  const float m_new = fmaxf(m_run, cmax);
  float alpha = 1.f;
  if (m_new > m_run) alpha = (m_run == NEG_INF) ? 0.f : ex2_approx(m_run - m_new);
  float pr[NS];
  float lsum = 0.f;
#pragma unroll
  for (int rs = 0; rs < NS; ++rs) {
    pr[rs] = (!FULL && sc[rs] == NEG_INF) ? 0.f : ex2_approx(sc[rs] - m_new);
    lsum += pr[rs];
  }
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
  l_run = l_run * alpha + lsum;
  m_run = m_new;
  if (__any_sync(0xffffffffu, alpha != 1.f)) {  // a row's max grew: rescale its sums
    // this lane accumulates rows 2q and 2q+1, whose factors sit in score lanes 8q and 8q+4
    const float a0 = __shfl_sync(0xffffffffu, alpha, 8 * sslot);
    const float a1 = __shfl_sync(0xffffffffu, alpha, 8 * sslot + 4);
#pragma unroll
    for (int u = 0; u < NT; ++u) {
      acc[u][0] *= a0; acc[u][2] *= a0;
      acc[u][1] *= a1; acc[u][3] *= a1;
    }
  }

  if constexpr (kCodeWords) {  // the V fields' codes
    using P = Preset<LP>;
    const uint4 r4 = *reinterpret_cast<const uint4*>(blk + P::FB + P::ORVQ);
    rq[0] = r4.x; rq[1] = r4.y; rq[2] = r4.z; rq[3] = r4.w;
    if constexpr (P::MASK) {
      const uint4 a4 = *reinterpret_cast<const uint4*>(blk + P::FB + P::OACT);
      ra[0] = a4.x; ra[1] = a4.y; ra[2] = a4.z; ra[3] = a4.w;
    }
  }

  // ---------------- values: O^T += V^T P^T on tensor cores ----------------
  // Round rr rebuilds tokens 4(rr*TPR + i) + slot (i < TPR) in lane (slot, j).  In the mma, A rows g
  // and g+8 (g = lane/4) of tile u are dims DPL*g + 2u and DPL*g + 2u + 1, B column g is query row
  // g, and k index 2q + e (q = lane%4; e < 2, then 8 + e for the k16 step) is the round's token
  // i = e (then 2 + e).  Lane (g, q) therefore takes the values rebuilt by lane (slot q, j g) =
  // 8q + g, pairs them by token with byte permutes, and supplies its own probabilities of those
  // tokens for row g (left in this lane by the score phase) split into fp16 hi + lo halves.
  // Two tokens per round: one m16n8k8 per tile; four: one m16n8k16.
  if constexpr (!DENSE && LP == kDs8PqOnly) {
    // PQ-only code tiles: lane (g, q) gathers V of its own k-pair tokens (4(rr*TPR + i) + q) at
    // subspace g (dims [8g, 8g+8)) straight from its codebook copy, so no shuffles are needed
    using P = Preset<LP>;
    const int g = lane >> 2;
    const uint16_t* cb = c.pq_vsel;
    const int pos = g ^ (2 * sslot);
#pragma unroll
    for (int rr = 0; rr < NR; ++rr) {
      uint32_t w[TPR][4];
#pragma unroll
      for (int i = 0; i < TPR; ++i) {
        const int tb = 4 * (rr * TPR + i) + sslot;
        const unsigned char* f = blk + (tb >> 4) * P::BLOCK + P::FB;
        const uint32_t code = f[P::OPQ + (tb & 15) * P::M + g];
        const uint4 v = *reinterpret_cast<const uint4*>(cb + ((code * P::M + pos) << 3));
        w[i][0] = v.x; w[i][1] = v.y; w[i][2] = v.z; w[i][3] = v.w;
      }
      uint32_t bhi[TPR / 2], blo[TPR / 2];
#pragma unroll
      for (int h = 0; h < TPR / 2; ++h) split_h2(pr[rr * TPR + 2 * h], pr[rr * TPR + 2 * h + 1], bhi[h], blo[h]);
#pragma unroll
      for (int u = 0; u < NT; ++u) {
        uint32_t a[TPR];
#pragma unroll
        for (int h = 0; h < TPR / 2; ++h) {
          a[2 * h] = prmt(w[2 * h][u], w[2 * h + 1][u], 0x5410u);
          a[2 * h + 1] = prmt(w[2 * h][u], w[2 * h + 1][u], 0x7632u);
        }
        if constexpr (TPR == 2) {
          mma16808(acc[u], a[0], a[1], bhi[0]);
          mma16808(acc[u], a[0], a[1], blo[0]);
        } else {
          mma16816(acc[u], a, bhi[0], bhi[1]);
          mma16816(acc[u], a, blo[0], blo[1]);
        }
      }
    }
    return;
  }
  const int src = (sslot << 3) | (lane >> 2);
#pragma unroll
  for (int rr = 0; rr < NR; ++rr) {
    int tb[TPR];
    bool valid[TPR];
#pragma unroll
    for (int i = 0; i < TPR; ++i) {
      tb[i] = 4 * (rr * TPR + i) + slot;
      valid[i] = FULL || (tb[i] >= t_lo && tb[i] < t_hi);
    }
    uint32_t w[TPR][DPL / 2];
    load_round<D, LP, DENSE, TPR, NB>(c, blk, dense_v, 1, tb, valid, t_lo, NR + rr, slot, j, dim0, odd, w, rq, ra,
                                      rr * TPR);
    uint32_t bhi[TPR / 2], blo[TPR / 2];
#pragma unroll
    for (int h = 0; h < TPR / 2; ++h) split_h2(pr[rr * TPR + 2 * h], pr[rr * TPR + 2 * h + 1], bhi[h], blo[h]);
#pragma unroll
    for (int u = 0; u < NT; ++u) {
      uint32_t a[TPR];
#pragma unroll
      for (int h = 0; h < TPR / 2; ++h) {
        const uint32_t x0 = __shfl_sync(0xffffffffu, w[2 * h][u], src);
        const uint32_t x1 = __shfl_sync(0xffffffffu, w[2 * h + 1][u], src);
        a[2 * h] = prmt(x0, x1, 0x5410u);      // dim DPL*g + 2u of the pair's two tokens
        a[2 * h + 1] = prmt(x0, x1, 0x7632u);  // dim DPL*g + 2u + 1
      }
      if constexpr (TPR == 2) {
        mma16808(acc[u], a[0], a[1], bhi[0]);
        mma16808(acc[u], a[0], a[1], blo[0]);
      } else {
        mma16816(acc[u], a, bhi[0], bhi[1]);
        mma16816(acc[u], a, blo[0], blo[1]);
      }
    }
  }
}

}  // namespace rfsn
