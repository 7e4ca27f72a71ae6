// decode_attn.cu — fused compressed-KV decode attention (flash-decoding split-K).
//
// Replaces RFSNv10KVCacheMLX.attention_forward (cache.py:395-428): the reference
// materialises the whole window in fp16 (materialize_window, cache.py:344-393,
// decoding warm/cold tokens with quantization.py:310-319) and then runs the
// fp32 blockwise online softmax of attention.py:39-105.  Here nothing is
// materialised: the window is streamed once from HBM.
//
// Work split.  Rows are (batch, kv-head) pairs; the window of every row is the
// same list of segments (hot dense run, warm code run, cold chunk runs).  The
// flattened (row, window-token) space is cut into equal contiguous ranges, one
// per CTA (one CTA per SM by default), so every SM streams the same number of
// tokens whatever the batch/head count.  A CTA emits one partial
// (max, sum, unnormalised output) per row it touches; rfsn_merge_kernel combines
// the partials of each row by log-sum-exp and writes fp16.
//
// Inside a CTA.  Warp NW (the producer, one elected lane) walks the CTA's tiles
// and issues 1-D bulk TMA copies (cp.async.bulk) of each tile's code streams
// (PQ, RVQ, RVQ-active, sparse idx/val) or hot fp16 K/V rows into a 3-stage
// shared-memory ring, signalling an mbarrier with the byte count.  Consumer
// warps 0..NW-1 take 8-token chunks of a tile; 8 lanes cooperate on one token,
// lane j owning dims [j*D/8, (j+1)*D/8).  For each token a lane rebuilds its
// dims exactly (fp16 PQ centroid + fp16 RVQ correction, fp16 add — see
// rfsn_decode.cuh) from codebooks staged in shared memory, forms partial dot
// products for every query row of the KV head (GQA group x queries), and the
// 8 partials are combined with xor-shuffles.  The top-S sparse residual enters
// K scores as q[idx]*val (fp32) and V outputs through a per-warp shared
// accumulator.  Softmax state is fp32 and rescaled only when a row's running
// max grows.  All waits are bounded (rfsn_common.cuh).
#include <cuda_runtime.h>
#include <math.h>

#include "rfsn_api_internal.h"
#include "rfsn_decode.cuh"

namespace rfsn {

constexpr int kStages = 3;
constexpr int kStageBytes = 32 * 1024;
constexpr int kNumFields = 10;  // k/v x {pq, rvq, mask, sp_idx, sp_val}
constexpr int kChunk = 8;       // tokens per warp chunk (2 row-steps of 4 tokens)
constexpr int64_t kMaxSmem = 227 * 1024;  // opt-in shared memory per CTA on sm_100

struct SegDev {
  int store, slot, first, count, pos0, wstart;
};

struct StoreDev {
  const uint8_t* f[5];  // pq, rvq, mask, sp_idx, sp_val
  int64_t cap, rows;
};

struct AttnParams {
  const uint16_t* q;
  const int32_t* qpos;
  float* ws_o;
  float* ws_ml;
  int32_t* dev_status;
  int B, Q, Hq, Hkv, D, G, R, causal;
  float scale;
  const uint16_t* hot_k;
  const uint16_t* hot_v;
  int64_t hot_cap;
  StoreDev sk[3], sv[3];  // index 1 = warm, 2 = cold pool
  const uint16_t* pq_cb;
  const uint16_t* rvq_cb;
  int M, K, ds, L, Kr, S, rvq_u16, has_mask;
  int64_t rows, W, per_cta;
  int max_pieces;
  int tile_codes, tile_dense;
  int field_bpt[kNumFields];   // bytes per token of each field (0 = absent)
  int field_base[kNumFields];  // byte offset of each field's region in a stage
  int nseg;
  int smem_pq, smem_rvq, smem_qtab, smem_vsp, smem_ml, smem_desc, smem_bar, smem_flag;
  SegDev seg[RFSN_MAX_SEGMENTS];
};

struct TileDesc {
  int kind;  // 0 = dense, 1 = compressed, -1 = done
  int n, pos0, row, first_of_piece, last_of_piece, piece, pad;
  int off[kNumFields];  // byte offset of each field's first token inside the stage
};

__device__ __forceinline__ void set_status(const AttnParams& p, volatile int* abort, int code) {
  *abort = 1;
  if (p.dev_status) atomicExch(p.dev_status, code);
}

// Bounded barrier among the NW consumer warps, built on an mbarrier (arrival
// count NW, one arrive per warp).  Returns false on timeout/abort.
__device__ __forceinline__ bool consumer_sync(uint64_t* bar, uint32_t& phase, volatile int* abort) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
  const bool ok = mbar_wait_bounded(bar, phase, abort);
  phase ^= 1u;
  __syncwarp();
  return ok;
}

template <int D, int RMAX, int NW, bool RVQ_SMEM>
__global__ void __launch_bounds__((NW + 1) * 32, 1) rfsn_decode_attn_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int DPL = D / 8;  // dims per lane
  constexpr int NG = DPL / 8;  // 8-dim groups per lane
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + p.smem_bar);
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* sync_bar = empty_bar + kStages;
  TileDesc* descs = reinterpret_cast<TileDesc*>(smem + p.smem_desc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + p.smem_flag);
  uint16_t* s_pq = reinterpret_cast<uint16_t*>(smem + p.smem_pq);
  uint16_t* s_rvq = reinterpret_cast<uint16_t*>(smem + p.smem_rvq);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], NW);
    }
    mbar_init(sync_bar, NW);
    *abort = 0;
    fence_mbar_init();
  }
  {  // stage codebooks
    const int n16 = p.M * p.K * p.ds / 8;
    for (int i = threadIdx.x; i < n16; i += blockDim.x)
      reinterpret_cast<uint4*>(s_pq)[i] = __ldg(reinterpret_cast<const uint4*>(p.pq_cb) + i);
    if (RVQ_SMEM && p.L > 0) {
      const int r16 = p.L * p.Kr * D / 8;
      for (int i = threadIdx.x; i < r16; i += blockDim.x)
        reinterpret_cast<uint4*>(s_rvq)[i] = __ldg(reinterpret_cast<const uint4*>(p.rvq_cb) + i);
    }
  }
  __syncthreads();

  const int64_t total = p.rows * p.W;
  const int64_t cta_a = (int64_t)blockIdx.x * p.per_cta;
  const int64_t cta_e = min(cta_a + p.per_cta, total);

  // ======================= producer warp =======================
  if (warp == NW) {
    if (lane != 0) return;
    int stage = 0;
    uint32_t phase = 0;
    bool inflight[kStages] = {};
    uint32_t inflight_parity[kStages] = {};
    bool ok = true;
    auto acquire = [&](int s) -> bool {
      if (!mbar_wait_bounded(&empty_bar[s], phase ^ 1u, abort)) {
        set_status(p, abort, kDevStatusTimeoutEmpty);
        return false;
      }
      return true;
    };
    auto advance = [&]() {
      if (++stage == kStages) {
        stage = 0;
        phase ^= 1u;
      }
    };
    for (int64_t a = cta_a; a < cta_e && ok;) {
      const int64_t row = a / p.W;
      const int64_t w0 = a - row * p.W;
      const int64_t w1 = min(p.W, w0 + (cta_e - a));
      const int piece = (int)(blockIdx.x - (row * p.W) / p.per_cta);
      bool first = true;
      for (int si = 0; si < p.nseg && ok; ++si) {
        const SegDev sg = p.seg[si];
        const int64_t s0 = max(w0, (int64_t)sg.wstart);
        const int64_t s1 = min(w1, (int64_t)sg.wstart + sg.count);
        if (s0 >= s1) continue;
        const int tile = sg.store == 0 ? p.tile_dense : p.tile_codes;
        for (int64_t t = s0; t < s1; t += tile) {
          const int n = (int)min((int64_t)tile, s1 - t);
          if (!acquire(stage)) {
            ok = false;
            break;
          }
          inflight[stage] = false;
          TileDesc* d = &descs[stage];
          unsigned char* sb = smem + (size_t)stage * kStageBytes;
          const int64_t tok = sg.first + (t - sg.wstart);
          for (int f = 0; f < kNumFields; ++f) d->off[f] = 0;
          d->n = n;
          d->pos0 = sg.pos0 + (int)(t - sg.wstart);
          d->row = (int)row;
          d->first_of_piece = first;
          d->last_of_piece = (t + n >= w1);
          d->piece = piece;
          first = false;
          uint32_t tx = 0;
          if (sg.store == 0) {
            d->kind = 0;
            const uint32_t bytes = (uint32_t)n * D * 2;
            const size_t src = ((size_t)row * p.hot_cap + tok) * D;
            d->off[0] = 0;
            d->off[1] = p.tile_dense * D * 2;
            tx = 2 * bytes;
            mbar_arrive_expect_tx(&full_bar[stage], tx);
            bulk_g2s(sb, p.hot_k + src, bytes, &full_bar[stage]);
            bulk_g2s(sb + d->off[1], p.hot_v + src, bytes, &full_bar[stage]);
          } else {
            d->kind = 1;
            const StoreDev& SK = p.sk[sg.store];
            const StoreDev& SV = p.sv[sg.store];
            const int64_t tindex = ((int64_t)sg.slot * SK.rows + row) * SK.cap + tok;
            uintptr_t lo[kNumFields];
            uint32_t len[kNumFields];
            for (int f = 0; f < kNumFields; ++f) {
              len[f] = 0;
              if (!p.field_bpt[f]) continue;
              const uint8_t* base = (f < 5 ? SK.f[f] : SV.f[f - 5]);
              const uintptr_t src = reinterpret_cast<uintptr_t>(base) + (uintptr_t)(tindex * p.field_bpt[f]);
              const uintptr_t l0 = src & ~(uintptr_t)15;
              const uintptr_t hi = (src + (uintptr_t)n * p.field_bpt[f] + 15) & ~(uintptr_t)15;
              lo[f] = l0;
              len[f] = (uint32_t)(hi - l0);
              d->off[f] = p.field_base[f] + (int)(src - l0);
              tx += len[f];
            }
            mbar_arrive_expect_tx(&full_bar[stage], tx);
            for (int f = 0; f < kNumFields; ++f)
              if (len[f]) bulk_g2s(sb + p.field_base[f], reinterpret_cast<const void*>(lo[f]), len[f], &full_bar[stage]);
          }
          inflight[stage] = true;
          inflight_parity[stage] = phase;
          advance();
        }
      }
      a += (w1 - w0);
    }
    if (ok && acquire(stage)) {
      descs[stage].kind = -1;
      mbar_arrive(&full_bar[stage]);
    } else {
      // Abort path: wait (bounded) for copies this thread issued so the CTA
      // never retires with bulk copies still writing its shared memory.
      for (int k = 0; k < kStages; ++k) {
        if (!inflight[k]) continue;
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&full_bar[k], inflight_parity[k])) {
          if (global_timer_ns() - t0 > kWaitLimitNs) break;
        }
      }
    }
    return;
  }

  // ======================= consumer warps =======================
  const int slot = lane >> 3;  // token slot within a row-step (0..3)
  const int j = lane & 7;      // dim group owner
  const int dim0 = j * DPL;
  float* qtab = reinterpret_cast<float*>(smem + p.smem_qtab) + (size_t)warp * D * RMAX;  // [D][RMAX]
  float* vsp = reinterpret_cast<float*>(smem + p.smem_vsp) + (size_t)warp * RMAX * D;    // [RMAX][D]
  float* s_ml = reinterpret_cast<float*>(smem + p.smem_ml);                              // [NW][RMAX][2]

  QzView qv;
  qv.pq_cb = s_pq;
  qv.rvq_cb = RVQ_SMEM ? s_rvq : p.rvq_cb;
  qv.M = p.M; qv.K = p.K; qv.ds = p.ds; qv.L = p.L; qv.Kr = p.Kr; qv.D = D; qv.S = p.S; qv.rvq_u16 = p.rvq_u16;
  const int rvq_bpt = p.L * (p.rvq_u16 ? 2 : 1);
  const float NEG_INF = __int_as_float(0xff800000);

  float qreg[RMAX][DPL];
  float acc[RMAX][DPL];
  float m_run[RMAX], l_run[RMAX];
  int qp[RMAX];
  int stage = 0;
  uint32_t phase = 0, sync_phase = 0;

  for (;;) {
    if (!mbar_wait_bounded(&full_bar[stage], phase, abort)) {
      set_status(p, abort, kDevStatusTimeoutFull);
      break;
    }
    const TileDesc desc = descs[stage];
    if (desc.kind < 0) break;
    const unsigned char* sb = smem + (size_t)stage * kStageBytes;
    const int row = desc.row;
    const int b = row / p.Hkv;
    const int kvh = row - b * p.Hkv;

    if (desc.first_of_piece) {
      // load this row's query rows (queries x GQA group) into registers / table
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        m_run[r] = NEG_INF;
        l_run[r] = 0.f;
        qp[r] = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          qreg[r][i] = 0.f;
          acc[r][i] = 0.f;
        }
        if (r < p.R) {
          const int qi = r / p.G, g = r - qi * p.G;
          const size_t qoff = ((size_t)(b * p.Q + qi) * p.Hq + kvh * p.G + g);
          const uint16_t* qsrc = p.q + qoff * D + dim0;
#pragma unroll
          for (int gg = 0; gg < NG; ++gg) {
            const uint4 w = *reinterpret_cast<const uint4*>(qsrc + 8 * gg);
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
            float f[8];
            unpack8(ww, f);
#pragma unroll
            for (int i = 0; i < 8; ++i) qreg[r][8 * gg + i] = f[i];
          }
          if (p.causal) qp[r] = p.qpos[qoff];
        }
      }
      for (int idx = lane; idx < D * RMAX; idx += 32) {
        const int d = idx / RMAX, r = idx - d * RMAX;
        float v = 0.f;
        if (r < p.R) {
          const int qi = r / p.G, g = r - qi * p.G;
          v = h2f(p.q[((size_t)(b * p.Q + qi) * p.Hq + kvh * p.G + g) * D + d]);
        }
        qtab[idx] = v;
        vsp[idx] = 0.f;
      }
      __syncwarp();
    }

    const int n = desc.n;
    const int nchunks = (n + kChunk - 1) / kChunk;
    for (int c = warp; c < nchunks; c += NW) {
      // ---------------- scores ----------------
      float sc[2][RMAX];
#pragma unroll
      for (int rs = 0; rs < 2; ++rs) {
        const int tl = c * kChunk + rs * 4 + slot;
        const bool valid = tl < n;
        float part[RMAX];
#pragma unroll
        for (int r = 0; r < RMAX; ++r) part[r] = 0.f;
        if (valid) {
#pragma unroll
          for (int gg = 0; gg < NG; ++gg) {
            uint32_t w[4];
            if (desc.kind == 0) {
              const uint4 v4 = *reinterpret_cast<const uint4*>(sb + desc.off[0] + ((size_t)tl * D + dim0 + 8 * gg) * 2);
              w[0] = v4.x; w[1] = v4.y; w[2] = v4.z; w[3] = v4.w;
            } else {
              const bool act = !p.has_mask || sb[desc.off[2] + tl] != 0;
              recon8(qv, sb + desc.off[0] + tl * p.M, sb + desc.off[1] + tl * rvq_bpt, act, dim0 + 8 * gg, w);
            }
            float f[8];
            unpack8(w, f);
#pragma unroll
            for (int r = 0; r < RMAX; ++r)
#pragma unroll
              for (int i = 0; i < 8; ++i) part[r] = __fmaf_rn(qreg[r][8 * gg + i], f[i], part[r]);
          }
          if (desc.kind == 1) {
            for (int e = j; e < p.S; e += 8) {
              const int idx = sb[desc.off[3] + tl * p.S + e];
              const float val = h2f(reinterpret_cast<const uint16_t*>(sb + desc.off[4])[tl * p.S + e]);
#pragma unroll
              for (int r = 0; r < RMAX; ++r) part[r] = __fmaf_rn(qtab[idx * RMAX + r], val, part[r]);
            }
          }
        }
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
          float v = part[r];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          const bool allowed = valid && r < p.R && (!p.causal || desc.pos0 + tl <= qp[r]);
          sc[rs][r] = allowed ? v * p.scale : NEG_INF;
        }
      }
      // ---------------- online softmax ----------------
      float pr[2][RMAX];
      bool grow = false;
      float alpha[RMAX];
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        float mx = fmaxf(sc[0][r], sc[1][r]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m_run[r], mx);
        alpha[r] = 1.f;
        if (m_new > m_run[r]) {
          alpha[r] = (m_run[r] == NEG_INF) ? 0.f : __expf(m_run[r] - m_new);
          grow = true;
          m_run[r] = m_new;
        }
        float ls = 0.f;
#pragma unroll
        for (int rs = 0; rs < 2; ++rs) {
          pr[rs][r] = (sc[rs][r] == NEG_INF) ? 0.f : __expf(sc[rs][r] - m_run[r]);
          ls += pr[rs][r];
        }
        ls += __shfl_xor_sync(0xffffffffu, ls, 8);
        ls += __shfl_xor_sync(0xffffffffu, ls, 16);
        // xor-8/16 sums over the 4 token slots of one dim-owner j: each token once
        l_run[r] = l_run[r] * alpha[r] + ls;
      }
      if (grow) {  // warp-uniform: m_run is replicated on all lanes
#pragma unroll
        for (int r = 0; r < RMAX; ++r)
#pragma unroll
          for (int i = 0; i < DPL; ++i) acc[r][i] *= alpha[r];
        for (int idx = lane; idx < RMAX * D; idx += 32) vsp[idx] *= alpha[idx / D];
        __syncwarp();
      }
      // ---------------- values ----------------
#pragma unroll
      for (int rs = 0; rs < 2; ++rs) {
        const int tl = c * kChunk + rs * 4 + slot;
        if (tl >= n) continue;
#pragma unroll
        for (int gg = 0; gg < NG; ++gg) {
          uint32_t w[4];
          if (desc.kind == 0) {
            const uint4 v4 = *reinterpret_cast<const uint4*>(sb + desc.off[1] + ((size_t)tl * D + dim0 + 8 * gg) * 2);
            w[0] = v4.x; w[1] = v4.y; w[2] = v4.z; w[3] = v4.w;
          } else {
            const bool act = !p.has_mask || sb[desc.off[7] + tl] != 0;
            recon8(qv, sb + desc.off[5] + tl * p.M, sb + desc.off[6] + tl * rvq_bpt, act, dim0 + 8 * gg, w);
          }
          float f[8];
          unpack8(w, f);
#pragma unroll
          for (int r = 0; r < RMAX; ++r)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[r][8 * gg + i] = __fmaf_rn(pr[rs][r], f[i], acc[r][8 * gg + i]);
        }
        if (desc.kind == 1) {
          for (int e = j; e < p.S; e += 8) {
            const int idx = sb[desc.off[8] + tl * p.S + e];
            const float val = h2f(reinterpret_cast<const uint16_t*>(sb + desc.off[9])[tl * p.S + e]);
#pragma unroll
            for (int r = 0; r < RMAX; ++r)
              if (r < p.R && pr[rs][r] != 0.f) atomicAdd(&vsp[r * D + idx], pr[rs][r] * val);
          }
        }
      }
    }
    // release the stage
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[stage]);

    if (desc.last_of_piece) {
      // reduce over the 4 token slots; fold in the sparse accumulator
#pragma unroll
      for (int r = 0; r < RMAX; ++r)
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          float v = acc[r][i];
          v += __shfl_xor_sync(0xffffffffu, v, 8);
          v += __shfl_xor_sync(0xffffffffu, v, 16);
          acc[r][i] = v;
        }
      __syncwarp();
      if (slot == 0) {
#pragma unroll
        for (int r = 0; r < RMAX; ++r)
#pragma unroll
          for (int i = 0; i < DPL; ++i) vsp[r * D + dim0 + i] += acc[r][i];
      }
      if (lane < RMAX) {
        s_ml[(warp * RMAX + lane) * 2 + 0] = m_run[lane];
        s_ml[(warp * RMAX + lane) * 2 + 1] = l_run[lane];
      }
      if (!consumer_sync(sync_bar, sync_phase, abort)) {
        set_status(p, abort, kDevStatusTimeoutFull);
        break;
      }
      // combine the NW warps' partials of this row
      const float* all_vsp = reinterpret_cast<const float*>(smem + p.smem_vsp);
      const size_t pbase = ((size_t)row * p.max_pieces + desc.piece) * p.R;
      for (int idx = threadIdx.x; idx < p.R * D; idx += NW * 32) {
        const int r = idx / D, d = idx - r * D;
        float M = NEG_INF;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, s_ml[(w * RMAX + r) * 2]);
        float O = 0.f, Ls = 0.f;
        if (M != NEG_INF) {
          for (int w = 0; w < NW; ++w) {
            const float mw = s_ml[(w * RMAX + r) * 2];
            if (mw == NEG_INF) continue;
            const float sc_w = __expf(mw - M);
            O = __fmaf_rn(all_vsp[(size_t)w * RMAX * D + r * D + d], sc_w, O);
            Ls = __fmaf_rn(s_ml[(w * RMAX + r) * 2 + 1], sc_w, Ls);
          }
        }
        p.ws_o[(pbase + r) * D + d] = O;
        if (d == 0) {
          p.ws_ml[(pbase + r) * 2 + 0] = M;
          p.ws_ml[(pbase + r) * 2 + 1] = Ls;
        }
      }
      if (!consumer_sync(sync_bar, sync_phase, abort)) {
        set_status(p, abort, kDevStatusTimeoutFull);
        break;
      }
    }
    if (++stage == kStages) {
      stage = 0;
      phase ^= 1u;
    }
  }
}

struct MergeParams {
  const float* ws_o;
  const float* ws_ml;
  uint16_t* out;
  int B, Q, Hq, Hkv, D, G, R, max_pieces;
  int64_t W, per_cta;
};

// One CTA per row: combine the row's partials by log-sum-exp and normalise
// (attention.py:104-105: a row whose every key is masked outputs zeros).
__global__ void rfsn_merge_kernel(const __grid_constant__ MergeParams p) {
  const int64_t row = blockIdx.x;
  const int64_t c0 = (row * p.W) / p.per_cta;
  const int64_t c1 = (row * p.W + p.W - 1) / p.per_cta;
  const int np = (int)(c1 - c0 + 1);
  const int b = (int)(row / p.Hkv), kvh = (int)(row % p.Hkv);
  const float NEG_INF = __int_as_float(0xff800000);
  for (int idx = threadIdx.x; idx < p.R * p.D; idx += blockDim.x) {
    const int r = idx / p.D, d = idx - r * p.D;
    float M = NEG_INF;
    for (int k = 0; k < np; ++k) M = fmaxf(M, p.ws_ml[(((size_t)row * p.max_pieces + k) * p.R + r) * 2]);
    float O = 0.f, L = 0.f;
    if (M != NEG_INF) {
      for (int k = 0; k < np; ++k) {
        const size_t pb = ((size_t)row * p.max_pieces + k) * p.R + r;
        const float mk = p.ws_ml[pb * 2];
        if (mk == NEG_INF) continue;
        const float s = __expf(mk - M);
        O = __fmaf_rn(p.ws_o[pb * p.D + d], s, O);
        L = __fmaf_rn(p.ws_ml[pb * 2 + 1], s, L);
      }
    }
    const float o = L > 0.f ? O / L : 0.f;
    const int qi = r / p.G, g = r - qi * p.G;
    p.out[(((size_t)b * p.Q + qi) * p.Hq + kvh * p.G + g) * p.D + d] = f2h(o);
  }
}

__global__ void rfsn_zero_kernel(uint16_t* out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = 0;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

struct Plan {
  AttnParams p;
  int nw, rmax;
  bool rvq_smem;
  int64_t smem;
  int grid;
  size_t ws_bytes;
};

// Consumer warps per CTA, chosen so the per-thread register budget of one
// CTA per SM covers q and the output accumulator without spilling.
static constexpr int consumer_warps(int D, int rmax) {
  return D == 64 ? (rmax == 1 ? 16 : rmax == 2 ? 12 : rmax == 4 ? 10 : 6) : (rmax == 1 ? 10 : rmax == 2 ? 8 : 6);
}

static int sm_count_cached() {
  static int count = 0;
  if (!count) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
    if (count <= 0) count = 148;
  }
  return count;
}

static void fill_store(StoreDev& d, const rfsn_code_store& s) {
  d.f[0] = s.pq;
  d.f[1] = reinterpret_cast<const uint8_t*>(s.rvq);
  d.f[2] = s.mask;
  d.f[3] = s.sp_idx;
  d.f[4] = reinterpret_cast<const uint8_t*>(s.sp_val);
  d.cap = s.cap;
  d.rows = s.rows;
}

static int make_plan(const rfsn_attn_args* a, const rfsn_quantizer* qz, Plan& pl) {
  int st = validate_quantizer(qz);
  if (st != RFSN_OK) return st;
  if (!a || !a->q || !a->out) return RFSN_ERR_INVALID_ARGUMENT;
  if (a->batch <= 0 || a->queries <= 0 || a->q_heads <= 0 || a->kv_heads <= 0) return RFSN_ERR_INVALID_ARGUMENT;
  if (a->q_heads % a->kv_heads) return RFSN_ERR_INVALID_ARGUMENT;
  if (a->head_dim != qz->head_dim) return RFSN_ERR_INVALID_ARGUMENT;
  if (a->head_dim != 64 && a->head_dim != 128) return RFSN_ERR_UNSUPPORTED;
  if (a->causal && !a->qpos) return RFSN_ERR_INVALID_ARGUMENT;
  if (a->num_segments < 0 || a->num_segments > RFSN_MAX_SEGMENTS) return RFSN_ERR_UNSUPPORTED;
  if (a->num_segments > 0 && !a->segments) return RFSN_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(a->q) & 15) || (reinterpret_cast<uintptr_t>(a->out) & 1)) return RFSN_ERR_ALIGNMENT;
  AttnParams& p = pl.p;
  p = AttnParams{};
  const int G = a->q_heads / a->kv_heads;
  const int R = G * a->queries;
  if (R > RFSN_MAX_ROWS_PER_KV) return RFSN_ERR_UNSUPPORTED;
  p.q = a->q; p.qpos = a->qpos; p.dev_status = a->device_status;
  p.B = a->batch; p.Q = a->queries; p.Hq = a->q_heads; p.Hkv = a->kv_heads; p.D = a->head_dim; p.G = G; p.R = R;
  p.causal = a->causal; p.scale = a->scale;
  p.hot_k = a->hot.k; p.hot_v = a->hot.v; p.hot_cap = a->hot.cap;
  fill_store(p.sk[1], a->warm_k); fill_store(p.sv[1], a->warm_v);
  fill_store(p.sk[2], a->cold_k); fill_store(p.sv[2], a->cold_v);
  p.pq_cb = qz->pq_codebooks; p.rvq_cb = qz->rvq_codebooks;
  p.M = qz->num_subspaces; p.K = qz->pq_codebook_size; p.ds = qz->subspace_dim; p.L = qz->rvq_layers;
  p.Kr = qz->rvq_codebook_size; p.S = qz->sparse_topk; p.rvq_u16 = qz->rvq_codebook_size > 256;
  p.has_mask = qz->rvq_layers > 0 && !(qz->rvq_threshold < 0.f);
  if (qz->rvq_layers > 8) return RFSN_ERR_UNSUPPORTED;
  p.rows = (int64_t)a->batch * a->kv_heads;

  // segments, validated against their stores (every token read must lie inside the store)
  int64_t W = 0;
  for (int i = 0; i < a->num_segments; ++i) {
    const rfsn_segment& s = a->segments[i];
    if (s.count < 0 || s.first < 0 || s.store < 0 || s.store > 2) return RFSN_ERR_INVALID_ARGUMENT;
    if (s.count == 0) continue;
    if (s.store == 0) {
      if (!a->hot.k || !a->hot.v || a->hot.cap <= 0 || a->hot.rows < p.rows) return RFSN_ERR_INVALID_ARGUMENT;
      if ((int64_t)s.first + s.count > a->hot.cap) return RFSN_ERR_INVALID_ARGUMENT;
      if ((reinterpret_cast<uintptr_t>(a->hot.k) & 15) || (reinterpret_cast<uintptr_t>(a->hot.v) & 15))
        return RFSN_ERR_ALIGNMENT;
    } else {
      const rfsn_code_store& ks = s.store == 1 ? a->warm_k : a->cold_k;
      const rfsn_code_store& vs = s.store == 1 ? a->warm_v : a->cold_v;
      if ((st = validate_store(&ks, qz)) != RFSN_OK) return st;
      if ((st = validate_store(&vs, qz)) != RFSN_OK) return st;
      if (ks.cap != vs.cap || ks.rows != vs.rows || ks.slots != vs.slots) return RFSN_ERR_INVALID_ARGUMENT;
      if (ks.rows < p.rows) return RFSN_ERR_INVALID_ARGUMENT;
      if (s.slot < 0 || s.slot >= ks.slots || (int64_t)s.first + s.count > ks.cap) return RFSN_ERR_INVALID_ARGUMENT;
    }
    if (p.nseg >= RFSN_MAX_SEGMENTS) return RFSN_ERR_UNSUPPORTED;
    SegDev& d = p.seg[p.nseg++];
    d.store = s.store; d.slot = s.slot; d.first = s.first; d.count = s.count; d.pos0 = s.pos0; d.wstart = (int)W;
    W += s.count;
  }
  if (W >= (int64_t)1 << 30) return RFSN_ERR_UNSUPPORTED;
  p.W = W;

  // per-token bytes of each compressed field and the stage layout
  const int rvq_bpt = qz->rvq_layers * (p.rvq_u16 ? 2 : 1);
  const int bpt[5] = {p.M, rvq_bpt, p.has_mask ? 1 : 0, p.S, p.S * 2};
  int per_token_bytes = 0;
  for (int f = 0; f < kNumFields; ++f) {
    p.field_bpt[f] = bpt[f % 5];
    per_token_bytes += p.field_bpt[f];
  }
  if (p.L == 0) p.field_bpt[1] = p.field_bpt[6] = 0;
  // compressed tile: largest multiple of 16 tokens (<= 256) whose regions fit a stage
  int tile = 256;
  for (; tile >= 16; tile -= 16) {
    int off = 0;
    for (int f = 0; f < kNumFields; ++f) {
      p.field_base[f] = off;
      if (p.field_bpt[f]) off += (int)align_up((int64_t)tile * p.field_bpt[f], 16) + 16;
    }
    if (off <= kStageBytes) break;
  }
  if (tile < 16) return RFSN_ERR_UNSUPPORTED;
  p.tile_codes = tile;
  p.tile_dense = kStageBytes / (2 * p.D * 2);  // 128 tokens for D=64, 64 for D=128
  (void)per_token_bytes;

  // kernel variant
  pl.rmax = R <= 1 ? 1 : R <= 2 ? 2 : R <= 4 ? 4 : 8;
  if (p.D == 128 && pl.rmax > 4) return RFSN_ERR_UNSUPPORTED;
  pl.nw = consumer_warps(p.D, pl.rmax);
  const int64_t pq_bytes = (int64_t)p.M * p.K * p.ds * 2;
  const int64_t rvq_bytes = (int64_t)p.L * p.Kr * p.D * 2;
  // Shared-memory layout; the RVQ codebook is staged only if it fits (else it
  // is read through L1/L2 from global memory).
  for (int attempt = 0; attempt < 2; ++attempt) {
    pl.rvq_smem = attempt == 0 && p.L > 0 && rvq_bytes <= 64 * 1024;
    int64_t off = (int64_t)kStages * kStageBytes;
    p.smem_pq = (int)off; off = align_up(off + pq_bytes, 128);
    p.smem_rvq = (int)off; if (pl.rvq_smem) off = align_up(off + rvq_bytes, 128);
    p.smem_qtab = (int)off; off = align_up(off + (int64_t)pl.nw * p.D * pl.rmax * 4, 128);
    p.smem_vsp = (int)off; off = align_up(off + (int64_t)pl.nw * pl.rmax * p.D * 4, 128);
    p.smem_ml = (int)off; off = align_up(off + (int64_t)pl.nw * pl.rmax * 2 * 4, 128);
    p.smem_desc = (int)off; off = align_up(off + (int64_t)kStages * sizeof(TileDesc), 128);
    p.smem_bar = (int)off; off = align_up(off + (2 * kStages + 1) * 8, 128);
    p.smem_flag = (int)off; off = align_up(off + 16, 128);
    pl.smem = off;
    if (pl.smem <= kMaxSmem) break;
  }
  if (pl.smem > kMaxSmem) return RFSN_ERR_UNSUPPORTED;

  // work split: equal contiguous ranges of the flattened (row, token) space
  const int64_t total = p.rows * W;
  int ctas = a->num_ctas > 0 ? a->num_ctas : sm_count_cached();
  if (total > 0) {
    int64_t per = (total + ctas - 1) / ctas;
    per = align_up(per, 16);
    p.per_cta = per;
    pl.grid = (int)((total + per - 1) / per);
    p.max_pieces = (int)((W + per - 1) / per) + 1;
  } else {
    p.per_cta = 1;
    pl.grid = 0;
    p.max_pieces = 1;
  }
  pl.ws_bytes = (size_t)p.rows * p.max_pieces * R * (p.D + 2) * sizeof(float) + 256;
  return RFSN_OK;
}

template <int D, int RMAX, int NW, bool RVQS>
static cudaError_t launch_variant(const Plan& pl, cudaStream_t s) {
  auto kern = rfsn_decode_attn_kernel<D, RMAX, NW, RVQS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
  if (e != cudaSuccess) return e;
  kern<<<pl.grid, (NW + 1) * 32, pl.smem, s>>>(pl.p);
  return cudaGetLastError();
}

template <int D, int RMAX, int NW>
static cudaError_t launch_rvq(const Plan& pl, cudaStream_t s) {
  return pl.rvq_smem ? launch_variant<D, RMAX, NW, true>(pl, s) : launch_variant<D, RMAX, NW, false>(pl, s);
}

static cudaError_t launch(const Plan& pl, cudaStream_t s) {
  const int D = pl.p.D;
  if (D == 64) {
    switch (pl.rmax) {
      case 1: return launch_rvq<64, 1, consumer_warps(64, 1)>(pl, s);
      case 2: return launch_rvq<64, 2, consumer_warps(64, 2)>(pl, s);
      case 4: return launch_rvq<64, 4, consumer_warps(64, 4)>(pl, s);
      default: return launch_rvq<64, 8, consumer_warps(64, 8)>(pl, s);
    }
  }
  switch (pl.rmax) {
    case 1: return launch_rvq<128, 1, consumer_warps(128, 1)>(pl, s);
    case 2: return launch_rvq<128, 2, consumer_warps(128, 2)>(pl, s);
    default: return launch_rvq<128, 4, consumer_warps(128, 4)>(pl, s);
  }
}

}  // namespace rfsn

using namespace rfsn;

extern "C" int rfsn_attention_workspace_size(const rfsn_attn_args* args, const rfsn_quantizer* qz, size_t* bytes) {
  if (!bytes) return RFSN_ERR_INVALID_ARGUMENT;
  Plan pl;
  const int st = make_plan(args, qz, pl);
  if (st != RFSN_OK) return st;
  *bytes = pl.ws_bytes;
  return RFSN_OK;
}

extern "C" int rfsn_decode_attention(const rfsn_attn_args* args, const rfsn_quantizer* qz, void* stream) {
  Plan pl;
  int st = make_plan(args, qz, pl);
  if (st != RFSN_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const AttnParams& p = pl.p;
  const int64_t nout = (int64_t)p.B * p.Q * p.Hq * p.D;
  if (p.W == 0) {
    rfsn_zero_kernel<<<(int)((nout + 255) / 256 < 1024 ? (nout + 255) / 256 : 1024), 256, 0, s>>>(args->out, nout);
    return check_cuda(cudaGetLastError());
  }
  if (!args->workspace || args->workspace_bytes < pl.ws_bytes) return RFSN_ERR_WORKSPACE_TOO_SMALL;
  if (reinterpret_cast<uintptr_t>(args->workspace) & 15) return RFSN_ERR_ALIGNMENT;
  pl.p.ws_ml = reinterpret_cast<float*>(args->workspace);
  pl.p.ws_o = pl.p.ws_ml + align_up((int64_t)p.rows * p.max_pieces * p.R * 2, 64);
  st = check_cuda(launch(pl, s));
  if (st != RFSN_OK) return st;
  MergeParams mp;
  mp.ws_o = pl.p.ws_o; mp.ws_ml = pl.p.ws_ml; mp.out = args->out;
  mp.B = p.B; mp.Q = p.Q; mp.Hq = p.Hq; mp.Hkv = p.Hkv; mp.D = p.D; mp.G = p.G; mp.R = p.R;
  mp.max_pieces = p.max_pieces; mp.W = p.W; mp.per_cta = p.per_cta;
  rfsn_merge_kernel<<<(int)p.rows, 256, 0, s>>>(mp);
  return check_cuda(cudaGetLastError());
}
