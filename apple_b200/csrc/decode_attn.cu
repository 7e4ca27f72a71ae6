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
// (max, sum, unnormalised output) per row piece it touches and then takes a
// ticket for the row; the CTA that completes a row's last piece combines the
// row's partials by log-sum-exp and writes fp16 (no separate merge launch).
// Tickets carry a launch tag in their upper 48 bits, so counts left by
// earlier or aborted launches are never taken for this launch's.  The tag is a
// launch counter kept at the start of the workspace: every CTA counts itself
// done on a second counter, and the last one resets that and advances the
// launch counter.  Replays of
// one captured launch (same kernel parameters) therefore get a fresh tag each
// time, and so does every launch of any shape that shares the workspace.
//
// Inside a CTA.  Warp NW (the producer) walks the CTA's tiles and issues 1-D
// bulk TMA copies (cp.async.bulk): a code tile is a run of whole 16-token
// blocks of the packed store (K and V fields interleaved, rfsn_layout.h), one
// contiguous copy; a hot tile is two copies (K rows, V rows).  Copies land in
// a shared-memory ring whose stages are guarded by full/empty mbarriers.
// Consumer warps 0..NW-1 take one 16-token block at a time (dealt
// round-robin); 8 lanes cooperate on one token, lane j owning dims
// [j*D/8, (j+1)*D/8).  A lane rebuilds its dims exactly from codebooks staged
// in shared memory (rfsn_attn_chunk.cuh), K scores for all query rows of the
// KV head (GQA group x queries) come from one tensor-core MMA per 8 dims, and
// P.V runs on tensor cores too (O^T = V^T P^T, fp32 accumulators).  Softmax state is fp32 and
// rescaled only when a row's running max grows.  All waits are bounded
// (rfsn_common.cuh).
#include <cuda_runtime.h>

#include <atomic>
#include <math.h>

#include <mutex>

#include "rfsn_api_internal.h"
#include "rfsn_attn_chunk.cuh"
#include "rfsn_attn_util.cuh"
#include "rfsn_decode.cuh"

namespace rfsn {

constexpr int kMaxStages = 8;                // mbarrier slots reserved per CTA
constexpr int kMaxStageBytes = 48 * 1024;    // upper bound of one ring stage
constexpr int kNoLimit = 1 << 30;         // position limit of a row that sees every token

// Tokens a consumer lane rebuilds per round (all loads in flight together) and
// the per-warp scratch that goes with it: two sets of sparse scatter rows
// [tokens per round][4 slots][D] fp16, reused as the warp's fp32 [RMAX][D]
// partial output when a piece ends.
// Layouts with a sparse residual or RVQ rows rebuild two tokens per round (four,
// measured on B200, ran 1.9x slower: the extra live registers cost more than the
// added load overlap).  PQ-only blocks rebuild a token with one gather, so they take
// four tokens per round for more independent loads and MMAs in flight; they have no
// sparse scatter rows, so the scratch size below (two tokens per round) still holds
// their fp32 partial output.
__host__ __device__ constexpr int tokens_per_round(int, int lp) { return lp == kDs8PqOnly ? 4 : 2; }
__host__ __device__ constexpr int scratch_bytes(int D) { return 2 * 2 * 4 * D * 2; }
// PQ-only blocks also take two blocks (32 tokens) per softmax update, halving the
// per-block cost of the max/sum shuffle chain; tiles then hold whole pairs.
__host__ __device__ constexpr int blocks_per_chunk(int lp) { return lp == kDs8PqOnly ? 2 : 1; }
constexpr int64_t kMaxSmem = 227 * 1024;  // opt-in shared memory per CTA on sm_100

struct SegDev {
  int store, slot, first, count, pos0, wstart;
};

struct StoreDev {
  const uint8_t* data;  // packed 16-token blocks (rfsn_layout.h)
  int64_t cap, rows;
};

struct AttnParams {
  const uint16_t* q;
  int64_t q_bstride;  // elements between consecutive sequences' queries
  const int32_t* qpos;
  uint16_t* out;
  float* ws_o;
  float* ws_ml;
  unsigned long long* tickets;  // one per row: (launch tag << 16) | pieces done
  unsigned long long* gen;      // [0] launch counter, [1] CTAs of this launch done (0 between launches)
  int32_t* dev_status;
  int B, Q, Hq, Hkv, D, G, R, causal;
  float scale;
  const uint16_t* hot_k;
  const uint16_t* hot_v;
  int64_t hot_cap;
  StoreDev st[3];  // index 1 = warm, 2 = cold pool
  BlockLayout lay;
  const uint16_t* pq_cb;
  const uint16_t* rvq_cb;
  int M, K, ds, L, Kr, S, rvq_u16, has_mask, rvq_smem;
  int64_t rows, W, per_cta;
  int max_pieces;
  int tile_blocks, tile_dense;  // code-tile length in 16-token blocks; dense-tile length in tokens
  int nseg;
  int smem_pq, smem_pqsw, smem_rvq, smem_scr, scr_bytes, smem_ml, smem_desc, smem_bar, smem_flag;
  int stages, stage_bytes, ring_off;  // ring depth, bytes per stage, ring offset in smem
  // fused output all-gather over peer memory (npeers == 0: off)
  int npeers, my_rank;
  int64_t seq_offset;  // this rank's first sequence in the gathered output
  int64_t full_elems;  // elements of one gathered-output buffer
  uint16_t* peer_buf[RFSN_MAX_PEERS];
  unsigned long long* peer_flags[RFSN_MAX_PEERS];
  unsigned long long* step;
  uint16_t* out_full;
  SegDev seg[RFSN_MAX_SEGMENTS];
};

struct TileDesc {
  int kind;  // 0 = dense, 1 = compressed, -1 = done
  int n, pos0, row, first_of_piece, last_of_piece, piece;
  int t0;    // compressed tiles: index of the first token inside the first copied block
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

// First and last CTA index whose token range touches row `row`: its pieces.
__device__ __forceinline__ int row_pieces(const AttnParams& p, int64_t row, int64_t* first_cta) {
  const int64_t c0 = (row * p.W) / p.per_cta;
  const int64_t c1 = (row * p.W + p.W - 1) / p.per_cta;
  *first_cta = c0;
  return (int)(c1 - c0 + 1);
}

// Log-sum-exp merge of a row's pieces (m in log2 units) and the fp16 output
// (attention.py:104-105: a row whose every key is masked outputs zeros).
// Flag words shared between GPUs.  The signalling thread fences once at system scope and then
// stores every rank's flag relaxed (a fence followed by relaxed stores releases everything
// before the fence); the waiting thread polls relaxed and fences once after it has seen every
// flag (relaxed loads followed by a fence acquire what the flags' writers released).
__device__ __forceinline__ void st_relaxed_sys(unsigned long long* a, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long* a) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}

// The launch's last CTA (gather mode): signal every rank that this rank's stores of the launch
// are done, wait (bounded) for every rank's signal, then copy the gathered output of this
// launch's parity into out_full.  `threads` consumer threads take part; thread 0 signals.
__device__ __noinline__ void gather_finish(const AttnParams& p, int parity, volatile int* abort, int threads) {
  volatile int* ok = abort + 3;
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned long long s = *reinterpret_cast<volatile unsigned long long*>(p.step) + 1ull;
    *reinterpret_cast<volatile unsigned long long*>(p.step) = s;
    for (int k = 0; k < p.npeers; ++k) st_relaxed_sys(p.peer_flags[k] + p.my_rank, s);  // after the fence above
    int good = 1;
    const unsigned long long* mine = p.peer_flags[p.my_rank];
    const uint64_t t0 = global_timer_ns();
    for (int r = 0; r < p.npeers && good; ++r) {
      for (uint32_t it = 0; ld_relaxed_sys(mine + r) < s; ++it) {
        if ((it & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
          good = 0;
          break;
        }
      }
    }
    if (good) __threadfence_system();  // acquires the peers' rows their flags released
    if (!good && p.dev_status) atomicExch(p.dev_status, kDevStatusPeerTimeout);
    *ok = good;
  }
  named_bar_sync(2, threads);
  if (!*ok) return;
  // the copy is latency-bound in one CTA: every thread keeps 8 loads in flight
  const uint4* src = reinterpret_cast<const uint4*>(p.peer_buf[p.my_rank] + (int64_t)parity * p.full_elems);
  uint4* dst = reinterpret_cast<uint4*>(p.out_full);
  const int64_t n = p.full_elems / 8;
  for (int64_t base = threadIdx.x; base < n; base += 8 * (int64_t)threads) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t i = base + (int64_t)u * threads;
      if (i < n) v[u] = __ldcg(src + i);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t i = base + (int64_t)u * threads;
      if (i < n) dst[i] = v[u];
    }
  }
}

// Gather mode: merge 8 consecutive dims of one query row per thread (the same fp32 operations
// per element, in the same order, as the scalar loop below) and store them as one 16-byte
// write to the local output and one to every rank's gathered-output buffer of this parity.
__device__ __noinline__ void merge_row_push(const AttnParams& p, int64_t row, int tid, int nthr, int parity) {
  int64_t c0;
  const int np = row_pieces(p, row, &c0);
  const int b = (int)(row / p.Hkv), kvh = (int)(row % p.Hkv);
  const float NEG_INF = __int_as_float(0xff800000);
  const int D8 = p.D / 8;
  for (int idx = tid; idx < p.R * D8; idx += nthr) {
    const int r = idx / D8, d = (idx - r * D8) * 8;
    float M = NEG_INF;
    for (int k = 0; k < np; ++k) M = fmaxf(M, __ldcg(&p.ws_ml[((row * p.max_pieces + k) * p.R + r) * 2]));
    float O[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, L = 0.f;
    if (M != NEG_INF) {
      for (int k = 0; k < np; ++k) {
        const int64_t pb = (row * p.max_pieces + k) * p.R + r;
        const float mk = __ldcg(&p.ws_ml[pb * 2]);
        if (mk == NEG_INF) continue;
        const float sc = ex2_approx(mk - M);
        const float4 o0 = __ldcg(reinterpret_cast<const float4*>(&p.ws_o[pb * p.D + d]));
        const float4 o1 = __ldcg(reinterpret_cast<const float4*>(&p.ws_o[pb * p.D + d + 4]));
        O[0] = __fmaf_rn(o0.x, sc, O[0]); O[1] = __fmaf_rn(o0.y, sc, O[1]);
        O[2] = __fmaf_rn(o0.z, sc, O[2]); O[3] = __fmaf_rn(o0.w, sc, O[3]);
        O[4] = __fmaf_rn(o1.x, sc, O[4]); O[5] = __fmaf_rn(o1.y, sc, O[5]);
        O[6] = __fmaf_rn(o1.z, sc, O[6]); O[7] = __fmaf_rn(o1.w, sc, O[7]);
        L = __fmaf_rn(__ldcg(&p.ws_ml[pb * 2 + 1]), sc, L);
      }
    }
    uint32_t h[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t lo = f2h(L > 0.f ? O[2 * e] / L : 0.f), hi = f2h(L > 0.f ? O[2 * e + 1] / L : 0.f);
      h[e] = lo | (hi << 16);
    }
    const uint4 v = make_uint4(h[0], h[1], h[2], h[3]);
    const int qi = r / p.G, g = r - qi * p.G;
    *reinterpret_cast<uint4*>(&p.out[(((size_t)b * p.Q + qi) * p.Hq + kvh * p.G + g) * p.D + d]) = v;
    const int64_t gi = (int64_t)parity * p.full_elems +
                       (((p.seq_offset + b) * p.Q + qi) * p.Hq + kvh * p.G + g) * (int64_t)p.D + d;
    for (int k = 0; k < p.npeers; ++k) *reinterpret_cast<uint4*>(p.peer_buf[k] + gi) = v;
  }
}

__device__ __forceinline__ void merge_row(const AttnParams& p, int64_t row, int tid, int nthr, int parity) {
  if (p.npeers) {
    merge_row_push(p, row, tid, nthr, parity);
    return;
  }
  int64_t c0;
  const int np = row_pieces(p, row, &c0);
  const int b = (int)(row / p.Hkv), kvh = (int)(row % p.Hkv);
  const float NEG_INF = __int_as_float(0xff800000);
  for (int idx = tid; idx < p.R * p.D; idx += nthr) {
    const int r = idx / p.D, d = idx - r * p.D;
    float M = NEG_INF;
    for (int k = 0; k < np; ++k) M = fmaxf(M, __ldcg(&p.ws_ml[((row * p.max_pieces + k) * p.R + r) * 2]));
    float O = 0.f, L = 0.f;
    if (M != NEG_INF) {
      for (int k = 0; k < np; ++k) {
        const int64_t pb = (row * p.max_pieces + k) * p.R + r;
        const float mk = __ldcg(&p.ws_ml[pb * 2]);
        if (mk == NEG_INF) continue;
        const float sc = ex2_approx(mk - M);
        O = __fmaf_rn(__ldcg(&p.ws_o[pb * p.D + d]), sc, O);
        L = __fmaf_rn(__ldcg(&p.ws_ml[pb * 2 + 1]), sc, L);
      }
    }
    const float o = L > 0.f ? O / L : 0.f;
    const int qi = r / p.G, g = r - qi * p.G;
    const uint16_t h = f2h(o);
    p.out[(((size_t)b * p.Q + qi) * p.Hq + kvh * p.G + g) * p.D + d] = h;
  }
}

template <int D, int RMAX, int NW, int LP>
__global__ void __launch_bounds__((NW + 1) * 32, 1) rfsn_decode_attn_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int DPL = D / 8;  // dims per lane
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + p.smem_bar);
  uint64_t* empty_bar = full_bar + kMaxStages;
  uint64_t* sync_bar = empty_bar + kMaxStages;
  TileDesc* descs = reinterpret_cast<TileDesc*>(smem + p.smem_desc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + p.smem_flag);
  uint16_t* s_pq = reinterpret_cast<uint16_t*>(smem + p.smem_pq);
  uint16_t* s_pqsw = reinterpret_cast<uint16_t*>(smem + p.smem_pqsw);  // 4-dim presets; PQ-only: 3 V copies
  uint16_t* s_rvq = reinterpret_cast<uint16_t*>(smem + p.smem_rvq);
  griddep_launch();  // a projection launched after this kernel may start streaming its weights

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], NW);
    }
    mbar_init(sync_bar, NW);
    *abort = 0;
    // gather mode: this launch's buffer parity (the last CTA advances the step afterwards)
    abort[2] = p.npeers ? (int)(*reinterpret_cast<volatile unsigned long long*>(p.step) & 1ull) : 0;
    abort[3] = 0;  // gather mode: set when this CTA stored a merged row to the peers
    fence_mbar_init();
  }
  __syncthreads();  // barriers initialised; the producer starts streaming at once
  if (warp < NW) {  // consumer warps stage the codebooks meanwhile
    // PQ codebook [M][K][ds] staged code-major [K][M][ds]: one code's centroids
    // for all subspaces form one row, so a token's lanes read distinct banks.
    // Consecutive threads write consecutive shared addresses (i = (c*M + m)*per + part).
    const int nc = p.M * p.K;
    const int nthr = NW * 32;
    if (p.ds % 8 == 0) {
      const int per = p.ds / 8;
      for (int i = threadIdx.x; i < nc * per; i += nthr) {
        const int cen = i / per, part = i - cen * per;
        const int c = cen / p.M, m = cen - c * p.M;
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.pq_cb) + (m * p.K + c) * per + part);
        reinterpret_cast<uint4*>(s_pq)[i] = v;
        if constexpr (LP == kDs8PqOnly) {
          // copies q = 1..3 for the V gathers of lanes with lane % 4 == q: subspace m at
          // position m ^ 2q, so a quarter-warp's 8 lanes hit 8 distinct bank groups
#pragma unroll
          for (int q = 1; q < 4; ++q) reinterpret_cast<uint4*>(s_pqsw)[(q - 1) * nc + c * 8 + (m ^ (2 * q))] = v;
        }
      }
    } else if (p.ds == 4) {
      // 4-dim presets also stage a copy with subspace pairs swapped (position m holds m^1)
      const bool sw = LP != kGeneric && Preset<LP>::DS == 4;
      for (int i = threadIdx.x; i < nc; i += nthr) {
        const int c = i / p.M, m = i - c * p.M;
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(p.pq_cb) + m * p.K + c);
        reinterpret_cast<uint2*>(s_pq)[i] = v;
        if (sw) reinterpret_cast<uint2*>(s_pqsw)[i ^ 1] = v;
      }
    } else {
      for (int i = threadIdx.x; i < nc * p.ds; i += nthr) {
        const int cen = i / p.ds, k = i - cen * p.ds;
        const int c = cen / p.M, m = cen - c * p.M;
        s_pq[i] = p.pq_cb[(m * p.K + c) * p.ds + k];
      }
    }
    if (p.rvq_smem && p.L > 0) {
      const int r16 = p.L * p.Kr * D / 8;
      for (int i = threadIdx.x; i < r16; i += nthr)
        reinterpret_cast<uint4*>(s_rvq)[i] = __ldg(reinterpret_cast<const uint4*>(p.rvq_cb) + i);
    }
    named_bar_sync(1, nthr);  // consumers only
  }

  // launch tag, read by the one thread that takes this CTA's tickets before any
  // CTA of the launch can advance the generation (that happens only after every
  // CTA has taken its done ticket, below)
  unsigned long long tag = 0;
  if (threadIdx.x == 0) tag = *reinterpret_cast<volatile unsigned long long*>(p.gen) & kTagMask;

  const int64_t total = p.rows * p.W;
  const int64_t cta_a = (int64_t)blockIdx.x * p.per_cta;
  const int64_t cta_e = min(cta_a + p.per_cta, total);

  // ======================= producer warp =======================
  // All 32 lanes walk the same tile sequence.  Lane 0 waits for a free stage,
  // writes the tile descriptor and arms the stage's mbarrier with the byte
  // count; then lane f issues the bulk copy of field f, so a tile's copies
  // enter the TMA unit in parallel instead of one after another.
  if (warp == NW) {
    int stage = 0;
    uint32_t phase = 0;
    uint32_t inflight = 0;         // bit s: stage s has copies issued
    uint32_t inflight_parity = 0;  // bit s: the phase parity those copies complete
    bool ok = true;
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
        for (int64_t t = s0; t < s1;) {
          const int64_t tok = sg.first + (t - sg.wstart);
          int n;
          if (sg.store == 0) {
            n = (int)min((int64_t)p.tile_dense, s1 - t);
          } else {  // whole 16-token blocks: the first may start mid-block
            n = (int)min((int64_t)p.tile_blocks * kBlockTokens - (tok % kBlockTokens), s1 - t);
          }
          int got = 1;
          if (lane == 0 && !mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, abort)) {
            set_status(p, abort, kDevStatusTimeoutEmpty);
            got = 0;
          }
          if (!__shfl_sync(0xffffffffu, got, 0)) {
            ok = false;
            break;
          }
          unsigned char* sb = smem + p.ring_off + (size_t)stage * p.stage_bytes;
          const void* my_src = nullptr;
          void* my_dst = nullptr;
          uint32_t my_len = 0;
          uint32_t tx = 0;
          int t0 = 0;
          if (sg.store == 0) {
            const uint32_t bytes = (uint32_t)n * D * 2;
            const size_t src = ((size_t)row * p.hot_cap + tok) * D;
            tx = 2 * bytes;
            if (lane < 2) {
              my_src = (lane == 0 ? p.hot_k : p.hot_v) + src;
              my_dst = sb + (lane == 0 ? 0 : p.tile_dense * D * 2);
              my_len = bytes;
            }
          } else {
            const StoreDev& SD = p.st[sg.store];
            const int64_t b0 = tok / kBlockTokens;
            const int64_t b1 = (tok + n + kBlockTokens - 1) / kBlockTokens;
            const int64_t blk = ((int64_t)sg.slot * SD.rows + row) * (SD.cap / kBlockTokens) + b0;
            t0 = (int)(tok - b0 * kBlockTokens);
            tx = (uint32_t)((b1 - b0) * p.lay.block_bytes);
            if (lane == 0) {
              my_src = SD.data + blk * p.lay.block_bytes;
              my_dst = sb;
              my_len = tx;
            }
          }
          if (lane == 0) {
            TileDesc* d = &descs[stage];
            d->kind = sg.store == 0 ? 0 : 1;
            d->n = n;
            d->pos0 = sg.pos0 + (int)(t - sg.wstart);
            d->row = (int)row;
            d->first_of_piece = first;
            d->last_of_piece = (t + n >= w1);
            d->piece = piece;
            d->t0 = t0;
            mbar_arrive_expect_tx(&full_bar[stage], tx);
          }
          t += n;
          first = false;
          __syncwarp();  // the barrier is armed before any copy can complete
          if (my_len) bulk_g2s(my_dst, my_src, my_len, &full_bar[stage]);
          inflight |= 1u << stage;
          inflight_parity = (inflight_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      a += (w1 - w0);
    }
    if (lane != 0) return;
    if (ok && mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, abort)) {
      descs[stage].kind = -1;
      mbar_arrive(&full_bar[stage]);
    } else {
      if (ok) set_status(p, abort, kDevStatusTimeoutEmpty);
      // Abort path: wait (bounded) for the copies issued into each stage so the
      // CTA never retires with bulk copies still writing its shared memory.
      for (int k = 0; k < p.stages; ++k) {
        if (!((inflight >> k) & 1u)) continue;
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&full_bar[k], (inflight_parity >> k) & 1u)) {
          if (global_timer_ns() - t0 > kWaitLimitNs) break;
        }
      }
    }
    return;
  }

  // ======================= consumer warps =======================
  // Lane (slot, j): slot = lane/8 is the token of a 4-token row-step, j = lane%8
  // owns dims [j*DPL, (j+1)*DPL).  K scores come from mma.m16n8k16 with the
  // lanes' reconstructed half2 registers as the B fragment (column = lane/4 =
  // (slot, dim half h = j/4), k = dims); A holds the query rows twice: rows
  // 0..7 matched to the h=0 dims, rows 8..15 to the h=1 dims.  Score(slot, r)
  // is then c0 + c3 of lane 4r + slot.  P.V runs on tensor cores as well
  // (O^T = V^T P^T, see process_block), so the output state is D/16 x 4 floats
  // per lane whatever the number of query rows.
  const int slot = lane >> 3;
  const int srow = lane >> 2;   // score lane: query row r
  const int sslot = lane & 3;   // score lane: token slot
  // per-warp scratch: fp16 sparse scatter rows while a piece runs, then the
  // warp's fp32 partial output [RMAX][D] when it ends
  unsigned char* scr = smem + p.smem_scr + (size_t)warp * p.scr_bytes;
  float* s_ml = reinterpret_cast<float*>(smem + p.smem_ml);  // [NW][RMAX][2]
  const float NEG_INF = __int_as_float(0xff800000);
  constexpr int NMMA = DPL / 4;  // K mma k-steps per row-step
  constexpr int kTpr = tokens_per_round(D, LP);
  constexpr int kNB = blocks_per_chunk(LP);     // 16-token blocks per softmax update
  constexpr int kChunk = kBlockTokens * kNB;
  constexpr int kBlock = LP != kGeneric ? Preset<LP>::BLOCK : 0;
  const int block_bytes = LP != kGeneric ? kBlock : p.lay.block_bytes;

  ChunkCtx c;
  c.pq_cm = s_pq;
  c.pq_sel = (Preset<LP>::DS == 4 && LP != kGeneric && (slot & 1)) ? s_pqsw : s_pq;
  c.pq_vsel = (LP == kDs8PqOnly && (lane & 3)) ? s_pqsw + (size_t)((lane & 3) - 1) * p.M * p.K * p.ds : s_pq;
  c.rvq_s = s_rvq;
  c.rvq_g = p.rvq_cb;
  c.scratch = reinterpret_cast<uint16_t*>(scr);
  c.lay = p.lay;
  c.M = p.M; c.K = p.K; c.ds = p.ds; c.L = p.L; c.Kr = p.Kr; c.S = p.S; c.rvq_u16 = p.rvq_u16;
  c.rvq_smem = p.rvq_smem; c.has_mask = p.has_mask;
  c.qp_lim = 0;
  c.sl2 = p.scale * 1.4426950408889634f;  // scores kept in log2 units
  uint32_t aq[NMMA][4];  // query A fragments
  float acc[D / 16][4];
  float m_run = NEG_INF, l_run = 0.f;  // online state of row srow (replicated over its 4 lanes)
  int stage = 0;
  uint32_t phase = 0, sync_phase = 0;
  int chunk_base = 0;  // global index of the current tile's first chunk

  for (;;) {
    if (!mbar_wait_bounded(&full_bar[stage], phase, abort)) {
      set_status(p, abort, kDevStatusTimeoutFull);
      break;
    }
    const TileDesc* dsc = &descs[stage];
    const int kind = dsc->kind;
    if (kind < 0) break;
    const int n = dsc->n;
    const int pos0 = dsc->pos0;
    const int row = dsc->row;
    const int first_of_piece = dsc->first_of_piece;
    const int last_of_piece = dsc->last_of_piece;
    const int piece = dsc->piece;
    const unsigned char* sb = smem + p.ring_off + (size_t)stage * p.stage_bytes;
    const int lead = kind == 0 ? 0 : dsc->t0;  // tokens of the first block that precede the tile
    const uint16_t* hot_k = reinterpret_cast<const uint16_t*>(sb);
    const uint16_t* hot_v = reinterpret_cast<const uint16_t*>(sb) + (size_t)p.tile_dense * D;
    const int b = row / p.Hkv;
    const int kvh = row - b * p.Hkv;

    if (first_of_piece) {
      m_run = NEG_INF;
      l_run = 0.f;
#pragma unroll
      for (int u = 0; u < D / 16; ++u) acc[u][0] = acc[u][1] = acc[u][2] = acc[u][3] = 0.f;
      {  // A fragments: lane (gA, tA) = (lane/4, lane%4); row gA is query row gA
        const int gA = lane >> 2, tA = lane & 3;
        const uint16_t* qrow = nullptr;
        if (gA < p.R) {
          const int qi = gA / p.G, g = gA - qi * p.G;
          qrow = p.q + (size_t)b * p.q_bstride + ((size_t)qi * p.Hq + kvh * p.G + g) * D;
        }
#pragma unroll
        for (int s = 0; s < NMMA; ++s) {
          const int dlo = tA * DPL + 4 * s, dhi = (4 + tA) * DPL + 4 * s;
          aq[s][0] = qrow ? ldg_u32(qrow + dlo) : 0u;
          aq[s][1] = qrow ? ldg_u32(qrow + dhi) : 0u;
          aq[s][2] = qrow ? ldg_u32(qrow + dlo + 2) : 0u;
          aq[s][3] = qrow ? ldg_u32(qrow + dhi + 2) : 0u;
        }
      }
      // last position row srow may see; rows past R see nothing
      c.qp_lim = srow < p.R ? kNoLimit : -kNoLimit;
      if (srow < p.R && p.causal) {
        const int qi = srow / p.G, g = srow - qi * p.G;
        c.qp_lim = p.qpos[(size_t)(b * p.Q + qi) * p.Hq + kvh * p.G + g];
      }
      for (int idx = lane; idx < p.scr_bytes / 16; idx += 32)
        reinterpret_cast<uint4*>(scr)[idx] = make_uint4(0u, 0u, 0u, 0u);
      __syncwarp();
    }

    // chunks (16-token blocks) are dealt round-robin over the CTA's whole tile
    // stream, so no warp carries an extra chunk of every tile
    const int span = lead + n;
    const int nchunks = (span + kChunk - 1) / kChunk;
    const int c_first = (warp - chunk_base % NW + NW) % NW;
    chunk_base += nchunks;
    for (int ch = c_first; ch < nchunks; ch += NW) {
      const int t_lo = ch == 0 ? lead : 0;
      const int t_hi = min(kChunk, span - ch * kChunk);
      const int pos_base = pos0 - lead + ch * kChunk;
      // a full chunk: all its tokens in range and visible to every live query row
      const bool full = t_lo == 0 && t_hi == kChunk &&
                        __all_sync(0xffffffffu, srow >= p.R || c.qp_lim >= pos_base + kChunk - 1);
      if (kind == 0) {
        const uint16_t* hk = hot_k + (size_t)ch * kChunk * D;
        const uint16_t* hv = hot_v + (size_t)ch * kChunk * D;
        if (full)
          process_block<D, RMAX, LP, true, kTpr, true, kNB>(c, nullptr, hk, hv, t_lo, t_hi, pos_base, aq, acc, m_run,
                                                            l_run);
        else
          process_block<D, RMAX, LP, true, kTpr, false, kNB>(c, nullptr, hk, hv, t_lo, t_hi, pos_base, aq, acc, m_run,
                                                             l_run);
      } else {
        const unsigned char* blk = sb + ch * kNB * block_bytes;
        if (full)
          process_block<D, RMAX, LP, false, kTpr, true, kNB>(c, blk, nullptr, nullptr, t_lo, t_hi, pos_base, aq, acc,
                                                             m_run, l_run);
        else
          process_block<D, RMAX, LP, false, kTpr, false, kNB>(c, blk, nullptr, nullptr, t_lo, t_hi, pos_base, aq, acc,
                                                              m_run, l_run);
      }
    }
    // release the stage
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[stage]);

    if (last_of_piece) {
      // lay the warp's partial out as [RMAX][D]: lane (g, q) holds rows 2q, 2q+1 at dims
      // DPL*g + 2u and DPL*g + 2u + 1
      float* part = reinterpret_cast<float*>(scr);
      {
        const int r0 = 2 * sslot, dg = srow * DPL;
#pragma unroll
        for (int u = 0; u < D / 16; ++u) {
          if (r0 < RMAX)
            *reinterpret_cast<float2*>(part + r0 * D + dg + 2 * u) = make_float2(acc[u][0], acc[u][2]);
          if (r0 + 1 < RMAX)
            *reinterpret_cast<float2*>(part + (r0 + 1) * D + dg + 2 * u) = make_float2(acc[u][1], acc[u][3]);
        }
      }
      if (sslot == 0 && srow < RMAX) {
        s_ml[(warp * RMAX + srow) * 2 + 0] = m_run;
        s_ml[(warp * RMAX + srow) * 2 + 1] = l_run;
      }
      if (!consumer_sync(sync_bar, sync_phase, abort)) {
        set_status(p, abort, kDevStatusTimeoutFull);
        break;
      }
      // combine the NW warps' partials of this row (m in log2 units)
      const size_t pbase = ((size_t)row * p.max_pieces + piece) * p.R;
      for (int idx = threadIdx.x; idx < p.R * D; idx += NW * 32) {
        const int r = idx / D, d = idx - r * D;
        float Mx = NEG_INF;
        for (int w = 0; w < NW; ++w) Mx = fmaxf(Mx, s_ml[(w * RMAX + r) * 2]);
        float O = 0.f, Ls = 0.f;
        if (Mx != NEG_INF) {
          for (int w = 0; w < NW; ++w) {
            const float mw = s_ml[(w * RMAX + r) * 2];
            if (mw == NEG_INF) continue;
            const float sc_w = ex2_approx(mw - Mx);
            const float* wp = reinterpret_cast<const float*>(smem + p.smem_scr + (size_t)w * p.scr_bytes);
            O = __fmaf_rn(wp[r * D + d], sc_w, O);
            Ls = __fmaf_rn(s_ml[(w * RMAX + r) * 2 + 1], sc_w, Ls);
          }
        }
        p.ws_o[(pbase + r) * D + d] = O;
        if (d == 0) {
          p.ws_ml[(pbase + r) * 2 + 0] = Mx;
          p.ws_ml[(pbase + r) * 2 + 1] = Ls;
        }
      }
      __threadfence();  // the partials are visible device-wide before the row ticket is taken
      if (!consumer_sync(sync_bar, sync_phase, abort)) {
        set_status(p, abort, kDevStatusTimeoutFull);
        break;
      }
      volatile int* merge_flag = abort + 1;
      if (warp == 0 && lane == 0) {
        int64_t c0;
        const int t = take_ticket(p.tickets + row, tag, row_pieces(p, row, &c0));
        if (t < 0) set_status(p, abort, kDevStatusTicket);
        *merge_flag = t > 0;
      }
      if (!consumer_sync(sync_bar, sync_phase, abort)) {
        set_status(p, abort, kDevStatusTimeoutFull);
        break;
      }
      if (*merge_flag) {  // this CTA finished the row: merge its pieces
        __threadfence();
        merge_row(p, row, threadIdx.x, NW * 32, abort[2]);
        if (p.npeers && threadIdx.x == 0) abort[3] = 1;
      }
    }
    if (++stage == p.stages) {
      stage = 0;
      phase ^= 1u;
    }
  }
  // Every CTA (also one that gave up on a timed-out wait) counts itself done; the
  // last one advances the launch counter, so the next launch on this workspace --
  // a graph replay with the same parameters included -- gets a new tag.
  // The done count is a plain counter that is zero between launches (the last CTA
  // resets it): one atomicAdd per CTA, where compare-and-swap tickets retried by
  // 148 CTAs finishing together serialise on round trips.
  if (p.npeers) {
    // A CTA that stored rows to the peers orders them before it counts itself done.  GPU scope
    // is enough here: the launch's last CTA observes this count, fences at system scope and then
    // releases the peers' flags, and that release carries every store ordered before it.
    named_bar_sync(2, NW * 32);
    if (abort[3]) __threadfence();
    named_bar_sync(2, NW * 32);
  }
  if (threadIdx.x == 0) {
    const bool last = atomicAdd(p.gen + 1, 1ull) == (unsigned long long)gridDim.x - 1ull;
    if (last) {
      atomicExch(p.gen + 1, 0ull);
      atomicAdd(p.gen, 1ull);
    }
    if (p.npeers) abort[1] = last;  // (the loop's merge flag: every consumer warp has left the loop)
  }
  if (p.npeers) {
    named_bar_sync(2, NW * 32);
    if (abort[1]) gather_finish(p, abort[2], abort, NW * 32);
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
  int nw, rmax, lp;
  bool rvq_smem;
  int64_t smem;
  int grid;
  size_t ws_bytes;
};

// Consumer warps per CTA, chosen so the per-thread register budget of one
// CTA per SM covers q and the output accumulator without spilling.  (Measured
// for PQ-only blocks on B200: one-block chunks at 19 warps / 96 registers ran
// 58.7 us per config-3 launch, two-block chunks at 15 warps / 128 registers
// 58.0 us; two-block chunks spill at 96 registers.)
static constexpr int consumer_warps(int D, int rmax, int lp) {
  if (D == 64 && lp == kDs8PqOnly) return 15;
  // total warps (NW + producer) a multiple of 4 so each SM sub-partition gets the same count
  // (the output state no longer depends on rmax; D = 128 keeps 16 dims per lane in flight)
  return D == 64 ? 15 : (rmax <= 2 ? 15 : 11);
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

// Compile-time layout preset for this configuration (kGeneric when none fits).
static int pick_preset(const AttnParams& p, bool rvq_smem) {
  if (p.D != 64 || p.K != 256) return kGeneric;
  if (p.L == 1 && (!rvq_smem || p.Kr != 256)) return kGeneric;
  int lp = kGeneric;
  if (p.ds == 4 && p.L == 1 && !p.has_mask && p.S == 8) lp = kDs4Rvq1DenseS8;
  else if (p.ds == 4 && p.L == 1 && p.has_mask && p.S == 0) lp = kDs4Rvq1Mask;
  else if (p.ds == 8 && p.L == 0 && p.S == 0) lp = kDs8PqOnly;
  else if (p.ds == 8 && p.L == 1 && p.has_mask && p.S == 0) lp = kDs8Rvq1Mask;
  bool ok = true;
  switch (lp) {
    case kDs4Rvq1DenseS8: ok = preset_layout_matches<kDs4Rvq1DenseS8>(p.lay); break;
    case kDs4Rvq1Mask: ok = preset_layout_matches<kDs4Rvq1Mask>(p.lay); break;
    case kDs8PqOnly: ok = preset_layout_matches<kDs8PqOnly>(p.lay); break;
    case kDs8Rvq1Mask: ok = preset_layout_matches<kDs8Rvq1Mask>(p.lay); break;
    default: break;
  }
  return ok ? lp : (int)kGeneric;
}

static void fill_store(StoreDev& d, const rfsn_code_store& s) {
  d.data = s.data;
  d.cap = s.cap;
  d.rows = s.rows;
}

static size_t workspace_layout(AttnParams& p, void* base);

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
  const int64_t q_packed = (int64_t)a->queries * a->q_heads * a->head_dim;
  if (a->q_batch_stride != 0 && (a->q_batch_stride < q_packed || (a->q_batch_stride & 7)))
    return RFSN_ERR_INVALID_ARGUMENT;
  p.q = a->q; p.qpos = a->qpos; p.dev_status = a->device_status;
  p.q_bstride = a->q_batch_stride ? a->q_batch_stride : q_packed;
  p.B = a->batch; p.Q = a->queries; p.Hq = a->q_heads; p.Hkv = a->kv_heads; p.D = a->head_dim; p.G = G; p.R = R;
  p.causal = a->causal; p.scale = a->scale;
  p.hot_k = a->hot.k; p.hot_v = a->hot.v; p.hot_cap = a->hot.cap;
  fill_store(p.st[1], a->warm);
  fill_store(p.st[2], a->cold);
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
      const rfsn_code_store& ks = s.store == 1 ? a->warm : a->cold;
      if ((st = validate_store(&ks, qz)) != RFSN_OK) return st;
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

  p.lay = layout_of(qz);
  // (tile sizes are chosen after the shared-memory layout fixes the stage size)
  // kernel variant
  pl.rmax = R <= 1 ? 1 : R <= 2 ? 2 : R <= 4 ? 4 : 8;
  const int64_t pq_bytes = (int64_t)p.M * p.K * p.ds * 2;
  const int64_t rvq_bytes = (int64_t)p.L * p.Kr * p.D * 2;
  // Shared-memory layout: codebooks and per-warp scratch first, the TMA ring
  // takes the rest (3 stages of up to 48 KB).  The RVQ codebook is staged only
  // if the ring keeps at least 3 x 24 KB (else it is read through L1/L2).
  // Per-warp scratch: 32*D bytes = fp16 sparse scatter rows [2][2][4][D], reused
  // for the warp's fp32 partial output [RMAX][D] (RMAX <= 8).
  p.stages = 3;
  p.scr_bytes = scratch_bytes(p.D);
  for (int attempt = 0; attempt < 2; ++attempt) {
    pl.rvq_smem = attempt == 0 && p.L > 0 && rvq_bytes <= 64 * 1024;
    pl.lp = pick_preset(p, pl.rvq_smem);
    pl.nw = consumer_warps(p.D, pl.rmax, pl.lp);
    const bool pq_swap = pl.lp == kDs4Rvq1DenseS8 || pl.lp == kDs4Rvq1Mask;
    int64_t off = 0;
    p.smem_pq = (int)off; off = align_up(off + pq_bytes, 128);
    p.smem_pqsw = (int)off;
    if (pq_swap) off = align_up(off + pq_bytes, 128);
    if (pl.lp == kDs8PqOnly) off = align_up(off + 3 * pq_bytes, 128);  // V-gather copies
    p.smem_rvq = (int)off; if (pl.rvq_smem) off = align_up(off + rvq_bytes, 128);
    p.smem_scr = (int)off; off = align_up(off + (int64_t)pl.nw * p.scr_bytes, 128);
    p.smem_ml = (int)off; off = align_up(off + (int64_t)pl.nw * pl.rmax * 2 * 4, 128);
    p.smem_desc = (int)off; off = align_up(off + (int64_t)kMaxStages * sizeof(TileDesc), 128);
    p.smem_bar = (int)off; off = align_up(off + (2 * kMaxStages + 1) * 8, 128);
    p.smem_flag = (int)off; off = align_up(off + 16, 128);
    const int64_t ring = ((kMaxSmem - off) / p.stages) / 1024 * 1024;
    p.stage_bytes = (int)(ring < kMaxStageBytes ? ring : kMaxStageBytes);
    pl.smem = off + (int64_t)p.stages * p.stage_bytes;
    if (p.stage_bytes >= 24 * 1024) break;
  }
  if (p.stage_bytes < 8 * 1024 || pl.smem > kMaxSmem) return RFSN_ERR_UNSUPPORTED;
  // the ring sits after the fixed regions
  p.ring_off = (int)(pl.smem - (int64_t)p.stages * p.stage_bytes);
  // compressed tile: the whole 16-token blocks that fit one stage (small blocks, e.g.
  // PQ-only codes at 256 B per block, make tiles of up to 192 blocks: every tile
  // costs a ring round trip, so tiles are as large as the stage allows)
  p.tile_blocks = p.stage_bytes / p.lay.block_bytes;
  if (p.tile_blocks > 1024) p.tile_blocks = 1024;
  p.tile_blocks -= p.tile_blocks % blocks_per_chunk(pl.lp);  // a chunk never reads past its stage
  if (p.tile_blocks < 2) return RFSN_ERR_UNSUPPORTED;
  p.tile_dense = (p.stage_bytes / (4 * p.D)) / 32 * 32;  // K and V rows of fp16, whole 32-token chunks
  if (p.tile_dense < 32) return RFSN_ERR_UNSUPPORTED;
  p.rvq_smem = pl.rvq_smem ? 1 : 0;
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
  if (p.max_pieces > 0xffff || pl.grid > 0xffff) return RFSN_ERR_UNSUPPORTED;  // tickets count in 16 bits
  if (a->gather) {  // fused output all-gather over peer memory
    const rfsn_peer_gather& g = *a->gather;
    if (g.num_ranks < 2 || g.num_ranks > RFSN_MAX_PEERS || g.rank < 0 || g.rank >= g.num_ranks || !g.step ||
        !g.out_full || g.seq_offset < 0 || g.seq_offset + a->batch > g.total_seqs)
      return RFSN_ERR_INVALID_ARGUMENT;
    // the merge stores 8 dims at a time: the local output and the buffers 16-byte aligned
    if ((reinterpret_cast<uintptr_t>(g.out_full) & 15) || (reinterpret_cast<uintptr_t>(a->out) & 15) ||
        (a->head_dim % 8))
      return RFSN_ERR_ALIGNMENT;
    for (int k = 0; k < g.num_ranks; ++k) {
      if (!g.buffers[k] || !g.flags[k]) return RFSN_ERR_INVALID_ARGUMENT;
      if ((reinterpret_cast<uintptr_t>(g.buffers[k]) & 15) || (reinterpret_cast<uintptr_t>(g.flags[k]) & 7))
        return RFSN_ERR_ALIGNMENT;
      p.peer_buf[k] = g.buffers[k];
      p.peer_flags[k] = reinterpret_cast<unsigned long long*>(g.flags[k]);
    }
    p.npeers = g.num_ranks;
    p.my_rank = g.rank;
    p.seq_offset = g.seq_offset;
    p.full_elems = g.total_seqs * a->queries * a->q_heads * a->head_dim;
    p.step = reinterpret_cast<unsigned long long*>(g.step);
    p.out_full = g.out_full;
  }
  pl.ws_bytes = workspace_layout(p, nullptr);
  return RFSN_OK;
}

// Workspace: a control region first -- the launch counter, the CTA done
// ticket and one 8-byte ticket per row, at the same offsets whatever the call's
// shape, so every launch that uses this workspace advances the one counter --
// then per (row, piece, query row) partial (max, sum) pairs and the
// unnormalised outputs.  Returns the bytes needed; with a base pointer, binds
// the regions into the parameters.
static size_t workspace_layout(AttnParams& p, void* base) {
  const int64_t ctl = align_up(16 + (int64_t)p.rows * 8, 256);
  const int64_t n_ml = align_up((int64_t)p.rows * p.max_pieces * p.R * 2, 64);
  const int64_t n_o = align_up((int64_t)p.rows * p.max_pieces * p.R * p.D, 64);
  if (base) {
    p.gen = reinterpret_cast<unsigned long long*>(base);
    p.tickets = p.gen + 2;
    p.ws_ml = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(base) + ctl);
    p.ws_o = p.ws_ml + n_ml;
  }
  return (size_t)ctl + (size_t)(n_ml + n_o) * sizeof(float);
}

template <int D, int RMAX, int NW, int LP>
static cudaError_t launch_variant(const Plan& pl, cudaStream_t s) {
  auto kern = rfsn_decode_attn_kernel<D, RMAX, NW, LP>;
  // the dynamic shared-memory limit is raised once per device to the largest size launched
  // (a per-launch attribute call costs host time on every decode step)
  static std::atomic<int> limit[64];
  int dev = -1;
  cudaGetDevice(&dev);
  const int need = (int)pl.smem;
  if (dev < 0 || dev >= 64 || need > limit[dev].load(std::memory_order_relaxed)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, need);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) {
      int cur = limit[dev].load(std::memory_order_relaxed);
      while (need > cur && !limit[dev].compare_exchange_weak(cur, need)) {
      }
    }
  }
  kern<<<pl.grid, (NW + 1) * 32, pl.smem, s>>>(pl.p);
  return cudaGetLastError();
}

template <int D, int RMAX, int NW>
static cudaError_t launch_ds(const Plan& pl, cudaStream_t s) {
  if constexpr (D == 64) {
    switch (pl.lp) {
      case kDs4Rvq1DenseS8: return launch_variant<D, RMAX, NW, kDs4Rvq1DenseS8>(pl, s);
      case kDs4Rvq1Mask: return launch_variant<D, RMAX, NW, kDs4Rvq1Mask>(pl, s);
      case kDs8PqOnly: return launch_variant<D, RMAX, consumer_warps(D, RMAX, kDs8PqOnly), kDs8PqOnly>(pl, s);
      case kDs8Rvq1Mask: return launch_variant<D, RMAX, NW, kDs8Rvq1Mask>(pl, s);
      default: break;
    }
  }
  return launch_variant<D, RMAX, NW, kGeneric>(pl, s);
}

static cudaError_t launch(const Plan& pl, cudaStream_t s) {
  const int D = pl.p.D;
  if (D == 64) {
    switch (pl.rmax) {
      case 1: return launch_ds<64, 1, consumer_warps(64, 1, kGeneric)>(pl, s);
      case 2: return launch_ds<64, 2, consumer_warps(64, 2, kGeneric)>(pl, s);
      case 4: return launch_ds<64, 4, consumer_warps(64, 4, kGeneric)>(pl, s);
      default: return launch_ds<64, 8, consumer_warps(64, 8, kGeneric)>(pl, s);
    }
  }
  switch (pl.rmax) {
    case 1: return launch_ds<128, 1, consumer_warps(128, 1, kGeneric)>(pl, s);
    case 2: return launch_ds<128, 2, consumer_warps(128, 2, kGeneric)>(pl, s);
    case 4: return launch_ds<128, 4, consumer_warps(128, 4, kGeneric)>(pl, s);
    default: return launch_ds<128, 8, consumer_warps(128, 8, kGeneric)>(pl, s);
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
  workspace_layout(pl.p, args->workspace);
  pl.p.out = args->out;
  return check_cuda(launch(pl, s));
}

// rfsn_decode_attention_host: the call with the query in host memory.  The query's
// bytes are copied into the caller's device staging buffer on the stream, the
// attention reads them from there, and with `synchronize` the call returns once
// the stream has finished, so an output in pinned (mapped) host memory, which the
// kernel writes over the bus, is then ready to read.
extern "C" int rfsn_decode_attention_host(const rfsn_attn_args* args, const rfsn_quantizer* qz,
                                          const uint16_t* q_host, uint16_t* q_stage, int synchronize, void* stream) {
  if (!args || !q_host || !q_stage) return RFSN_ERR_INVALID_ARGUMENT;
  if (args->batch <= 0 || args->queries <= 0 || args->q_heads <= 0 || args->head_dim <= 0)
    return RFSN_ERR_INVALID_ARGUMENT;
  if (args->q_batch_stride != 0 &&
      args->q_batch_stride != (int64_t)args->queries * args->q_heads * args->head_dim)
    return RFSN_ERR_INVALID_ARGUMENT;  // the staged query is packed
  const size_t bytes = (size_t)args->batch * args->queries * args->q_heads * args->head_dim * sizeof(uint16_t);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(q_stage, q_host, bytes, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return check_cuda(e);
  rfsn_attn_args a = *args;
  a.q = q_stage;
  const int st = rfsn_decode_attention(&a, qz, stream);
  if (st != RFSN_OK || !synchronize) return st;
  return check_cuda(cudaStreamSynchronize(s));
}

// ---------------------------------------------------------------------------
// rfsn_decode_attention_noalloc: the same attention with partials kept in a
// fixed module-scope buffer instead of a caller-provided workspace.
//
// Some callers cannot allocate device memory at the moment they run decode
// attention: a host-language binding that holds only q/out/store pointers and
// has no device allocator of its own, or an embedding runtime whose memory is
// reserved up front and may not grow per call.  For them the split-K partials
// (max, sum and unnormalised output of every row piece) live in a static
// __device__ array of kNoAllocScratchBytes per device.  Its address is looked
// up once per device, on the first call made with that device current, and
// cached; that first call may load the module, so make it before capturing
// the stream into a graph.  Nothing here calls an allocator.  Every partial
// the merge reads is written by the attention kernel of the same call, and the
// per-row completion tickets carry each launch's own tag (a launch counter in
// the buffer that every launch advances; the buffer starts zeroed like every
// __device__ array), so values left by earlier (or aborted) calls are never
// counted: the buffer needs no clearing between calls.  Calls that
// overlap in time on one device
// (different streams, or threads without ordering) share the buffer and race;
// calls on one stream are ordered and safe.
// ---------------------------------------------------------------------------
namespace rfsn {

constexpr size_t kNoAllocScratchBytes = RFSN_NOALLOC_SCRATCH_BYTES;  // 4 MiB per device
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[kNoAllocMaxDevices];

// Device address of this device's scratch (looked up on first use).
static int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return check_cuda(e);
  if (dev < 0 || dev >= kNoAllocMaxDevices) return RFSN_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
    if (e != cudaSuccess) return check_cuda(e);
    if (!addr) return RFSN_ERR_CUDA;
    g_noalloc_ptr[dev] = addr;
  }
  *out = g_noalloc_ptr[dev];
  return RFSN_OK;
}

}  // namespace rfsn

extern "C" int rfsn_decode_attention_noalloc(const rfsn_attn_args* args, const rfsn_quantizer* qz, void* stream) {
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
  // partials of all row pieces must fit the fixed buffer
  if (pl.ws_bytes > kNoAllocScratchBytes) return RFSN_ERR_WORKSPACE_TOO_SMALL;
  void* scratch = nullptr;
  st = noalloc_scratch(&scratch);
  if (st != RFSN_OK) return st;
  workspace_layout(pl.p, scratch);
  pl.p.out = args->out;
  return check_cuda(launch(pl, s));
}
